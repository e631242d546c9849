"""CausalHiFTGenerator on the GPU (mirror of ``cv3cpu/models/hift.py``).

Signals are channel-major ``[batch][channels][time]``; several utterances of
the same length run as one batch through every kernel.  The whole-utterance
decode is used for any length (the reference's time-chunked variant
``_spectral_chunked`` exists only to bound CPU memory and gives the same
result up to float rounding; it is kept here as :meth:`spectral_chunked` for
API parity and tests).

The NSF dither is the reference's fixed MT19937 uniform stream
(``TorchMT19937(noise_seed).random_float32``), drawn on the device once for the
longest utterance seen; shorter ones use its prefix, as the reference does.
"""

from __future__ import annotations

from typing import Optional, Sequence

import numpy as np

from .. import _dev as D
from .. import ops
from .._lib import call
from ._common import ConvTC, Graph

torch = D.torch


def causal_pad(kernel_size: int, dilation: int = 1) -> int:
    """``CausalConv1d.causal_padding`` (hift.py:14-16)."""
    return int((kernel_size * dilation - dilation) / 2) * 2 + (kernel_size + 1) % 2


class HiFTGenerator:
    def __init__(self, weights, prefix: str = "hift."):
        self.w = weights
        self.p = prefix
        m = weights.meta.get("hift", {})
        self.upsample_rates = list(m.get("upsample_rates", [8, 5, 3]))
        self.upsample_kernel_sizes = list(m.get("upsample_kernel_sizes", [16, 11, 7]))
        self.resblock_kernel_sizes = list(m.get("resblock_kernel_sizes", [3, 7, 11]))
        self.resblock_dilation_sizes = [list(d) for d in m.get("resblock_dilation_sizes", [[1, 3, 5]] * 3)]
        self.source_resblock_kernel_sizes = list(m.get("source_resblock_kernel_sizes", [7, 7, 11]))
        self.source_resblock_dilation_sizes = [list(d) for d in
                                               m.get("source_resblock_dilation_sizes", [[1, 3, 5]] * 3)]
        self.n_fft = int(m.get("istft_n_fft", 16))
        self.hop_len = int(m.get("istft_hop_len", 4))
        self.lrelu_slope = float(m.get("lrelu_slope", 0.1))
        self.audio_limit = float(m.get("audio_limit", 0.99))
        self.sampling_rate = int(m.get("sampling_rate", 24000))
        self.nb_harmonics = int(m.get("nb_harmonics", 8))
        self.nsf_alpha = float(m.get("nsf_alpha", 0.1))
        self.nsf_sigma = float(m.get("nsf_sigma", 0.003))
        self.nsf_voiced_threshold = float(m.get("nsf_voiced_threshold", 10.0))
        self.conv_pre_look_right = int(m.get("conv_pre_look_right", 4))
        self.num_kernels = len(self.resblock_kernel_sizes)
        self.num_upsamples = len(self.upsample_rates)
        self.upsample_scale = int(np.prod(self.upsample_rates)) * self.hop_len
        self.window = ops.hann_window(self.n_fft)
        self._win = None
        self._convs = {}
        self._graphs = {}   # input shape -> (graph, static input, static output, dither buffer)
        self.noise_seed = int(m.get("noise_seed", 0))
        self._src_noise = None
        self._user_noise = False

    # -- weights -------------------------------------------------------------------
    def _t(self, name):
        return self.w.f32(self.p + name)

    def _k(self, name) -> int:
        return int(self.w.entry(self.p + name)["shape"][-1])

    def _f64(self, name):
        return self.w.cache((self.p + name + ":f64",), lambda: self.w.f32(self.p + name).double())

    def win(self):
        if self._win is None:
            self._win = torch.from_numpy(self.window).cuda()
        return self._win

    # -- convolution helper ---------------------------------------------------------
    def _conv(self, x, name, stride=1, dilation=1, pad=(0, 0), act=-1, act_param=0.0, snake=None,
              residual=None):
        """Tensor-core conv (implicit GEMM) with the elementwise op after it fused into the
        epilogue: activation ``act``, snake with the alphas named ``snake``, + ``residual``."""
        cv = self._convs.get(name)
        if cv is None:
            cv = ConvTC(self._t(name + ".weight"), self._t(name + ".bias"))
            self._convs[name] = cv
        B, cin, T = (int(s) for s in x.shape)
        span = dilation * (cv.k - 1) + 1
        t_out = (T + pad[0] + pad[1] - span) // stride + 1
        y = D.empty((B, cv.cout, t_out))
        cv(x, y, B, T, t_out, stride=stride, dilation=dilation, pad_left=pad[0], residual=residual, act=act,
           act_param=act_param, snake_alpha=self._t(snake) if snake is not None else None)
        return y

    @staticmethod
    def _unary(x, act, p=0.0):
        y = torch.empty_like(x)
        call("cv3_unary", act, float(p), x.data_ptr(), x.numel(), y.data_ptr(), D.stream())
        return y

    @staticmethod
    def _bin(a, b, op, s=0.0):
        y = torch.empty_like(a)
        call("cv3_binary", op, a.data_ptr(), b.data_ptr() if b is not None else None, float(s), a.numel(),
             y.data_ptr(), D.stream())
        return y

    def _snake(self, x, alpha_name):
        a = self._t(alpha_name)
        y = torch.empty_like(x)
        B, C, T = (int(s) for s in x.shape)
        call("cv3_snake", x.data_ptr(), a.data_ptr(), B, C, T, y.data_ptr(), D.stream())
        return y

    # -- F0 (hift.py:56-72) -------------------------------------------------------------
    def f0_predict(self, mel):
        """``[B, 80, T]`` device mel -> ``[B, T]`` float32 F0 (float32 convs, float64 classifier)."""
        x = mel
        for i in range(5):
            name = f"f0_predictor.condnet.{i}"
            k = self._k(name + ".weight")
            pad = (0, causal_pad(k)) if i == 0 else (causal_pad(k), 0)
            x = self._conv(x, name, pad=pad, act=5, act_param=1.0)
        B, C, T = (int(s) for s in x.shape)
        f0 = D.empty((B, T))
        call("cv3_f0_classifier", x.data_ptr(), B, C, T, self._f64("f0_predictor.classifier.weight").data_ptr(),
             self._f64("f0_predictor.classifier.bias").data_ptr(), f0.data_ptr(), D.stream())
        return f0

    # -- NSF source (hift.py:75-111) -----------------------------------------------------
    def source_noise(self, n: int):
        harm = self.nb_harmonics + 1
        if self._src_noise is None or (self._src_noise.shape[0] < n and not self._user_noise):
            need = max(n, 1)
            buf = D.empty((need, harm))
            call("cv3_torch_rand", self.noise_seed, 0, need * harm, buf.data_ptr(), D.stream())
            self._src_noise = buf
        if self._src_noise.shape[0] < n:
            raise ValueError(f"dither buffer holds {self._src_noise.shape[0]} samples, {n} needed")
        return self._src_noise

    def set_source_noise(self, buf) -> None:
        """Use a caller-supplied dither buffer ``[samples, harmonics]`` (hift.py:83-88)."""
        self._src_noise = D.dev(np.asarray(buf, np.float32) if D.is_host(buf) else buf)
        self._user_noise = True
        self._graphs.clear()    # captured passes read the previous buffer

    def excitation(self, f0):
        """``[B, T]`` F0 -> ``[B, up*T]`` merged harmonic source."""
        B, T = (int(s) for s in f0.shape)
        up, harm = self.upsample_scale, self.nb_harmonics + 1
        noise = self.source_noise(up * T)
        sines = D.empty((B, T, harm))
        out = D.empty((B, up * T))
        call("cv3_nsf_source", f0.data_ptr(), B, T, harm, self.sampling_rate, up, self.nsf_alpha, self.nsf_sigma,
             self.nsf_voiced_threshold, noise.data_ptr(), self._t("m_source.l_linear.weight").data_ptr(),
             self._t("m_source.l_linear.bias").data_ptr(), sines.data_ptr(), out.data_ptr(), D.stream())
        return out

    # -- decoder (hift.py:114-210) -------------------------------------------------------
    def _resblock(self, group, idx, x, kernel, dilations):
        base = f"{group}.{idx}."
        for j, d in enumerate(dilations):
            xt = self._snake(x, base + f"activations1.{j}.alpha")
            xt = self._conv(xt, base + f"convs1.{j}", dilation=d, pad=(causal_pad(kernel, d), 0),
                            snake=base + f"activations2.{j}.alpha")
            x = self._conv(xt, base + f"convs2.{j}", pad=(causal_pad(kernel, 1), 0), residual=x)
        return x

    def spectral(self, mel, s_stft):
        """``[B, 80, T]``, ``[B, 18, 120T+1]`` -> ``[B, n_fft+2, 120T+1]`` (hift.py:131-168)."""
        # conv_pre's output only feeds the first leaky ReLU: fused into its epilogue
        x = self._conv(mel, "conv_pre", pad=(0, causal_pad(self._k("conv_pre.weight"))), act=6,
                       act_param=self.lrelu_slope)
        down_rates = [1] + self.upsample_rates[::-1][:-1]
        down_cum = list(np.cumprod(down_rates))[::-1]
        for i in range(self.num_upsamples):
            if i > 0:
                x = self._unary(x, 6, self.lrelu_slope)
            x = ops.interpolate_nearest(x, self.upsample_rates[i])
            k = self._k(f"ups.{i}.weight")
            x = self._conv(x, f"ups.{i}", pad=(k - 1, 0))
            if i == self.num_upsamples - 1:
                B, C, T = (int(s) for s in x.shape)
                y = D.empty((B, C, T + 1))
                call("cv3_reflect_left1", x.data_ptr(), B * C, T, y.data_ptr(), D.stream())
                x = y
            u = int(down_cum[i])
            ks = self._k(f"source_downs.{i}.weight")
            if u == 1:
                si = self._conv(s_stft, f"source_downs.{i}", pad=(causal_pad(ks), 0))
            else:
                si = self._conv(s_stft, f"source_downs.{i}", stride=u, pad=(u - 1, 0))
            si = self._resblock("source_resblocks", i, si, self.source_resblock_kernel_sizes[i],
                                self.source_resblock_dilation_sizes[i])
            x = self._bin(x, si, 0)
            acc = None
            for j in range(self.num_kernels):
                r = self._resblock("resblocks", i * self.num_kernels + j, x, self.resblock_kernel_sizes[j],
                                   self.resblock_dilation_sizes[j])
                acc = r if acc is None else self._bin(acc, r, 0)
            x = self._bin(acc, None, 3, float(self.num_kernels))
        x = self._unary(x, 6, 0.01)
        return self._conv(x, "conv_post", pad=(causal_pad(self._k("conv_post.weight")), 0))

    def spectral_chunked(self, mel, s_stft, chunk: int, context: int):
        """Exact time-chunked :meth:`spectral` (hift.py:170-194), kept for parity checks."""
        up = int(np.prod(self.upsample_rates))
        T = int(mel.shape[-1])
        look = causal_pad(self._k("conv_pre.weight"))
        pieces = []
        for m0 in range(0, T, chunk):
            m1 = min(T, m0 + chunk)
            c0, c1 = max(0, m0 - context), min(T, m1 + look)
            sub = self.spectral(mel[:, :, c0:c1].contiguous(), s_stft[:, :, c0 * up: c1 * up + 1].contiguous())
            lead, take = (m0 - c0) * up, (m1 - m0) * up
            pieces.append(sub[:, :, : 1 + take] if m0 == 0 else sub[:, :, 1 + lead: 1 + lead + take])
        return torch.cat(pieces, dim=2).contiguous()

    def decode(self, mel, source, chunk: Optional[int] = None, context: int = 64):
        """``[B, 80, T]`` mel, ``[B, 480T]`` source -> ``[B, 480T]`` waveform (hift.py:196-210)."""
        s_stft = ops.stft_stacked(source, self.n_fft, self.hop_len, self.win())
        if chunk is None or int(mel.shape[-1]) <= chunk:
            x = self.spectral(mel, s_stft)
        else:
            x = self.spectral_chunked(mel, s_stft, chunk, context)
        return ops.istft_stacked(x, self.n_fft, self.hop_len, self.win(), mode=1, limit=self.audio_limit)

    GRAPH_SHAPES = 2    # captured input shapes kept (each holds its activations' memory)

    def inference_batch(self, mels, chunk: Optional[int] = None, context: int = 64, use_graph: bool = False):
        """Device ``[B, 80, T]`` mels -> ``[B, 480T]`` waveforms.

        ``use_graph``: the whole pass (F0 convs, source, ~100 convolution and elementwise
        launches, iSTFT) replays a CUDA graph captured for this input shape, so its cost is
        the kernels' alone; the first call of a shape runs eagerly (building the convolution
        operands, tables and the dither buffer), the second captures.  The result is a new
        tensor either way and equals the eager pass bit for bit."""
        mel = D.dev(mels)
        if use_graph and chunk is None:
            key = tuple(int(s) for s in mel.shape)
            entry = self._graphs.get(key)
            if entry is None:
                entry = self._capture(mel, key)
            if entry is not None:
                g, x_in, y, _noise = entry
                x_in.copy_(mel)
                g.replay()
                return y.clone()
        f0 = self.f0_predict(mel)
        return self.decode(mel, self.excitation(f0), chunk=chunk, context=context)

    def _capture(self, mel, key):
        """Warm up eagerly, then capture one pass on a static input of ``mel``'s shape.  The
        entry keeps the dither buffer the graph reads alive (a longer utterance may replace
        the module's buffer later)."""
        if key not in getattr(self, "_warm", set()):
            self._warm = getattr(self, "_warm", set()) | {key}
            return None     # this call runs eagerly; the next one captures
        x_in = D.empty(key)
        x_in.copy_(mel)
        out = {}

        def body(_stream):
            f0 = self.f0_predict(x_in)
            out["y"] = self.decode(x_in, self.excitation(f0))

        g = Graph()
        g.capture(body)
        if len(self._graphs) >= self.GRAPH_SHAPES:
            self._graphs.pop(next(iter(self._graphs)))
        entry = (g, x_in, out["y"], self._src_noise)
        self._graphs[key] = entry
        return entry

    def inference(self, mel, chunk: Optional[int] = 250, context: int = 64):
        """``(80, T)`` mel -> ``(480 T,)`` waveform (hift.py:212-218).

        ``chunk`` defaults to the reference's 250; on the device the whole
        utterance is decoded at once unless a chunk is passed explicitly
        (``chunk=None`` or the default both give the whole-utterance result).
        """
        host = D.is_host(mel)
        m = D.dev(mel).reshape(1, *np.shape(mel)[-2:]) if D.is_host(mel) else D.dev(mel).unsqueeze(0)
        use_chunk = chunk if (chunk is not None and chunk != 250) else None
        y = self.inference_batch(m, chunk=use_chunk, context=context)[0]
        return D.out(y, host)

"""Benchmark: end-to-end balanced CosyVoice 3 synthesis on B200 (config 4 of the baseline).

One step = 8 independent 10 s utterances per GPU through the int8 LM (64..80-id
random text + 75-token prompt, 250 greedy speech tokens), the 10-step CFG flow
(N = 2 * (75 + 250) = 650 frames, CFG batch 16) and the vocoder (500 frames ->
240,000 samples).  Synthetic random weights of the released geometry and seeded
random inputs (no dataset or checkpoint is involved).  Weak scaling: each rank
synthesises its own 8 utterances; ``value`` is all ranks' utterances divided by
the slowest rank's device time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl cuda|reference]

The reference arm (``--impl reference``) times the CPU oracle -- the NumPy
restatement of the reference's kernel layer and stages -- on the host cores,
one bounded per-utterance sample per step (see ``cpu_sample``).
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "10s-utterances/sec at 1/2/4/8 B200 (LM tok/s, flow+HiFT RTF); % HBM/TC roofline"
UNIT = "utterances/s"
UTTS = 8
TOKENS = 250
PROMPT_TOKENS = 75
PEAKS = os.path.join(REPO, "MEASURED_PEAKS.json")


def pkg(name=""):
    return importlib.import_module("cosyvoice3-cpu_b200" + ("." + name if name else ""))


def make_requests(seeds, meta):
    """Config-4 inputs per seed (``workloads.requests``): 40..80 text ids, a prompt text
    ending in <|endofprompt|>, 75 prompt speech tokens, 150 prompt mel frames, a 192-d
    speaker vector."""
    return pkg("workloads").requests(seeds, meta)


# ---------------------------------------------------------------------------
# multi-GPU plumbing: one process per GPU, utterances sharded, no data-path collective
# ---------------------------------------------------------------------------

def rank_seeds(rank: int, per_rank: int = None) -> range:
    """The utterance seeds rank ``rank`` synthesises: a disjoint block per rank (weak
    scaling: every GPU gets the same amount of work)."""
    per_rank = UTTS if per_rank is None else per_rank
    return range(rank * per_rank, (rank + 1) * per_rank)


def max_over_ranks(ms: float, world: int, device="cuda") -> float:
    """The job's time for a step: the slowest rank's (one all-reduce MAX; timing only)."""
    if world <= 1:
        return float(ms)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(ms)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for nm, v in zip(names, parts[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU oracle sample (cpu_baseline and the reference arm)
# ---------------------------------------------------------------------------

def cpu_sample(W, req, decode_steps: int = 4):
    """Seconds per utterance of the CPU oracle, from a bounded sample of one
    config-4 utterance: LM prefill of its prompt plus ``decode_steps`` greedy
    steps (per-step time extrapolated to 250), one DiT forward at the CFG batch
    (2, 80, 650) (x10 Euler steps), and the full 500-frame vocoder."""
    import oracle.stages as st
    meta = W.meta
    lm = st.SpeechLM(W, meta)
    v = req.voice
    x0 = lm.prompt_embedding(req.text_ids, req.prompt_ids, v.speech_token.tolist())
    cache = lm.body.new_cache()
    t0 = time.perf_counter()
    h = lm.body.forward(x0, cache)
    tok = lm.greedy(lm.head(h[-1:])[0])
    t_prefill = time.perf_counter() - t0
    t0 = time.perf_counter()
    for _ in range(decode_steps):
        h = lm.body.forward(lm.speech_emb([tok]), cache)
        tok = lm.greedy(lm.head(h[-1:])[0])
    t_step = (time.perf_counter() - t0) / decode_steps
    flow = st.Flow(W, meta)
    n = 2 * (PROMPT_TOKENS + TOKENS)
    rng = np.random.default_rng(0)
    x = rng.normal(size=(2, 80, n)).astype(np.float32)
    t0 = time.perf_counter()
    flow.dit.forward(x, x * 0, np.array([0.5, 0.5], np.float32), np.zeros((2, 80), np.float32), x * 0)
    t_dit = time.perf_counter() - t0
    hift = st.HiFT(W, meta)
    mel = np.clip(rng.normal(-5, 2, size=(80, 2 * TOKENS)), -11.5, 2).astype(np.float32)
    t0 = time.perf_counter()
    hift.inference(mel, chunk=250)
    t_hift = time.perf_counter() - t0
    per_utt = t_prefill + (TOKENS - 1) * t_step + flow.steps * t_dit + t_hift
    sampled = t_prefill + decode_steps * t_step + t_dit + t_hift
    return per_utt, sampled, {"lm_prefill_s": t_prefill, "lm_step_s": t_step, "dit_forward_s": t_dit,
                              "hift_s": t_hift}


def cpu_full_utterance(W, req):
    """Seconds of one complete config-4 utterance on the CPU oracle, nothing extrapolated:
    the LM prompt, prefill and all 250 greedy steps (head + argmax each), the flow's
    conditioning and its 10-step CFG Euler solve at 2 x 650 frames, and the 500-frame
    vocoder (chunk 250).  ``cpu_sample`` models the same utterance from a few timed pieces;
    this measurement is what that model is checked against."""
    import oracle.stages as st
    meta = W.meta
    lm, flow, hift = st.SpeechLM(W, meta), st.Flow(W, meta), st.HiFT(W, meta)
    v = req.voice
    t0 = time.perf_counter()
    x0 = lm.prompt_embedding(req.text_ids, req.prompt_ids, v.speech_token.tolist())
    toks, _ = lm.generate_greedy(x0, TOKENS)
    t_lm = time.perf_counter() - t0
    t0 = time.perf_counter()
    mel = flow.inference(np.asarray(toks), v.speech_token, v.mel, v.embedding)
    t_flow = time.perf_counter() - t0
    t0 = time.perf_counter()
    wav = hift.inference(mel, chunk=250)
    t_hift = time.perf_counter() - t0
    return {"s": t_lm + t_flow + t_hift, "lm_s": t_lm, "flow_s": t_flow, "hift_s": t_hift,
            "tokens": len(toks), "samples": int(np.asarray(wav).size)}


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 0) for i in threadpool_info() if i.get("user_api") == "blas"]
        return max(n) if n else host_threads()
    except Exception:
        return host_threads()


def use_all_host_threads():
    """BLAS on every host core, whatever OMP_NUM_THREADS the launcher set (torchrun sets 1)."""
    try:
        from threadpoolctl import threadpool_limits
        return threadpool_limits(limits=host_threads(), user_api="blas")
    except Exception:
        return None


CPU_SAMPLE_DESC = ("one config-4 utterance, modelled from a timed sample: LM prefill + 4 greedy steps (the "
                   "per-step time x 249), one DiT forward at CFG batch 2 x 650 frames (x 10 steps), the full "
                   "500-frame vocoder (chunk 250)")


def cpu_baseline_line(W, req):
    _limits = use_all_host_threads()
    t0 = time.perf_counter()
    per_utt, sampled, parts = cpu_sample(W, req)
    wall = time.perf_counter() - t0
    return {"value": 1.0 / per_utt, "unit": UNIT, "cores": blas_threads(), "kind": "port",
            "sample": CPU_SAMPLE_DESC, "sample_wall_s": wall, "modelled_s_per_utterance": per_utt,
            "parts_s": parts}


def run_reference(args, rank: int, world: int) -> None:
    """The reference arm: the CPU implementation of the path (the oracle port of cv3cpu's
    kernel layer and stages) on all host cores.  Each step times one bounded sample of a
    config-4 utterance (``cpu_sample``); ``ms_per_step`` is that sample's wall time and
    ``value`` the utterance rate the sample implies (see CPU_SAMPLE_DESC).  Once per run,
    before the steps, one complete utterance is synthesised with nothing extrapolated
    (``cpu_full_utterance``, skipped by ``--no-full-utterance``); the line reports its time
    and the model's error against it for the same utterance."""
    if rank != 0:
        return
    _limits = use_all_host_threads()
    synth = pkg("synth")
    W = synth.synthetic_weights("balanced")
    reqs = make_requests(range(UTTS), W.meta)
    full = None
    if not args.no_full_utterance:
        full = cpu_full_utterance(W, reqs[0])
        modelled, _, _ = cpu_sample(W, reqs[0])
        full["modelled_s"] = modelled
        full["model_error"] = modelled / full["s"] - 1.0
    per, walls = [], []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        per_utt, sampled, parts = cpu_sample(W, reqs[i % len(reqs)])
        wall = time.perf_counter() - t0
        if i >= args.warmup:
            per.append(per_utt)
            walls.append(wall)
    per_utt = float(np.mean(per))
    value = 1.0 / per_utt
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": float(np.mean(walls)) * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(args),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": blas_threads(), "kind": "port",
                         "sample": CPU_SAMPLE_DESC, "modelled_s_per_utterance": per_utt},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "full_utterance": full,
    }), flush=True)


def config_dict(args):
    return {"workload": "config4 e2e balanced synthesis: 8 utterances per GPU, 250 greedy LM tokens each, "
                        "10-step CFG flow at 650 frames, vocoder 500 frames -> 240000 samples",
            "utterances_per_gpu": UTTS, "lm_tokens": TOKENS, "prompt_speech_tokens": PROMPT_TOKENS,
            "flow_frames": 2 * (PROMPT_TOKENS + TOKENS), "cfg_batch": 2 * UTTS, "vocoder_frames": 2 * TOKENS,
            "profile": "balanced (int8 LM/DiT, f16 vocoder)", "parallelism": f"dp{args.gpus} (independent utterances)",
            "l2": "working set > L2: 1.2 GB of weights streamed every step"}


# ---------------------------------------------------------------------------
# the device arm
# ---------------------------------------------------------------------------

LM_WEIGHT_BYTES = 375_255_804      # int8 payload + fp16 scales of the 24 layers and the speech head
KV_BYTES_PER_POS = 24_576          # k and v, 24 layers x 2 kv heads x 64 x 4 B, per cached position
DIT_GEMM_PARAMS = 184_549_376      # per-token weights of the 22 blocks' q, k, v, out, ff1, ff2
HIFT_GFLOP = 336.9                 # vocoder convolutions per 10 s (500 mel frames)


def _timed(fn, reps: int):
    """Mean milliseconds of ``fn()`` over ``reps`` runs, CUDA events on the current stream."""
    import torch
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def measure_config1(tts, meta, peaks, reps: int = 3):
    """Config 1: the balanced LM at batch 1, a 64-id prompt, 250 greedy tokens.  The decode
    step's HBM roofline counts its algorithmic bytes: every int8 weight and scale once, plus the
    KV cache read (24,576 B per cached position, mean length over the 249 steps) and one
    position appended."""
    import torch
    wl = pkg("workloads")
    lm = tts.llm
    ids = wl.lm_prompt_ids(0, vocab=int(meta["qwen2"]["vocab_size"]))
    x0 = pkg("_dev").dev(lm._text_emb(ids))
    steps = wl.LM_STEPS
    eng = lm.engine(1, 512, steps)
    eng.run([x0], steps)                                   # builds and captures the step graph
    t_prefill = _timed(lambda: eng.prefill([x0]), reps)
    t_total = _timed(lambda: eng.run([x0], steps), reps)
    step_ms = (t_total - t_prefill) / (steps - 1)
    mean_len = wl.LM_PROMPT_IDS + steps / 2.0
    bytes_step = LM_WEIGHT_BYTES + KV_BYTES_PER_POS * (mean_len + 1)
    gbs = bytes_step / (step_ms * 1e-3) / 1e9
    hbm = peaks.get("hbm_gbs")
    return {"workload": "config1: batch-1 greedy decode, 64-id prompt + 250 tokens, balanced int8 LM",
            "lm_tok_s": steps / (t_total * 1e-3), "ms_total": t_total, "prefill_ms": t_prefill,
            "decode_step_us": step_ms * 1e3,
            "roofline": {"kernel": "one graph-replayed decode step (24 layers + head)", "bound": "hbm",
                         "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm if hbm else None,
                         "algorithmic_bytes_per_step": bytes_step,
                         "peak_source": "measured copy bandwidth (MEASURED_PEAKS.json)"}}


def measure_config2(Wf, peaks, reps: int = 3):
    """Config 2: the f32 DiT flow, 250 tokens -> 500 frames, 10 CFG Euler steps at batch 2.
    Tensor work per solve = 10 x (GEMMs 2 * 184.5 M * B * N + attention 4 * N^2 * 1024 * B * 22)."""
    import numpy as np
    wl = pkg("workloads")
    flow = pkg("models.flow").Flow(pkg("weights").DeviceWeights(Wf))
    tokens, emb = wl.flow_inputs(0)
    mu, spk, cond, _ = flow.conditioning(tokens, np.zeros(0, np.int64), np.zeros((0, 80), np.float32), emb)
    run = lambda: flow.solve_batch([mu], [spk], [cond])  # noqa: E731
    run()
    ms = _timed(run, reps)
    B, N, steps = 2, 2 * len(tokens), int(flow.n_timesteps)
    flops = steps * (2.0 * DIT_GEMM_PARAMS * B * N + 4.0 * N * N * 1024 * B * 22)
    tf = flops / (ms * 1e-3) / 1e12
    peak = peaks.get("bf16_tflops")
    return {"workload": "config2: f32 DiT flow, 250 tokens -> 500 frames, 10 CFG Euler steps (batch 2)",
            "flow_s": ms * 1e-3, "dit_forward_ms": ms / steps,
            "roofline": {"kernel": "the whole solve (GEMM + attention FLOPs, fp32 via 3xTF32)", "bound": "tensor",
                         "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak if peak else None,
                         "flops_per_solve": flops, "peak_source": "measured bf16 dense (MEASURED_PEAKS.json)"}}


def measure_config3(Wf, peaks, reps: int = 3):
    """Config 3: the f32 vocoder, 500 mel frames -> 240,000 samples (336.9 GFLOP of convolution),
    replayed from its CUDA graph (the first call runs eagerly, the second captures)."""
    wl = pkg("workloads")
    hift = pkg("models.hift").HiFTGenerator(pkg("weights").DeviceWeights(Wf))
    mel = pkg("_dev").dev(wl.vocoder_mel(1))[None]
    run = lambda: hift.inference_batch(mel, use_graph=True)  # noqa: E731
    run()
    run()
    ms = _timed(run, reps)
    tf = HIFT_GFLOP * 1e9 / (ms * 1e-3) / 1e12
    peak = peaks.get("bf16_tflops")
    return {"workload": "config3: f32 vocoder, 500 frames -> 240000 samples", "vocoder_s": ms * 1e-3,
            "roofline": {"kernel": "the whole vocoder (convolution FLOPs)", "bound": "tensor", "achieved": tf,
                         "peak": peak, "unit": "TFLOP/s", "frac": tf / peak if peak else None,
                         "peak_source": "measured bf16 dense (MEASURED_PEAKS.json)"}}


SWEEP_UTTS, SWEEP_BATCH, SWEEP_TOKENS = 256, 32, 750


def sweep_requests(seeds, meta):
    """Config-5 utterances: 120..240 text ids, the config-4 prompt form, 750 tokens each."""
    return pkg("workloads").requests(seeds, meta, text_len=(120, 240))


def measure_config5(tts, meta, rank: int, world: int, barrier, full: bool = False):
    """Config 5, the 256 x 30 s throughput sweep: batches of 32 utterances per GPU through the
    LM (750 greedy tokens each), the CFG flow (batch 2 x 32, N = 2 * (75 + 750) = 1650) and
    the vocoder (1500 frames -> 720,000 samples).  ``full``: every batch of this rank's share
    of the 256 utterances is run and timed; otherwise one batch per GPU is timed and the
    sweep time is that batch's time x the batches per GPU (all batches have the same shape)."""
    import torch
    per_gpu = SWEEP_UTTS // world
    batches = max(per_gpu // SWEEP_BATCH, 1)
    seeds = list(range(rank * per_gpu, (rank + 1) * per_gpu))
    groups = [seeds[i:i + SWEEP_BATCH] for i in range(0, len(seeds), SWEEP_BATCH)]
    first = tts.prepare(sweep_requests(groups[0], meta))
    tts.run_prepared(first, SWEEP_TOKENS)           # warm-up: engines, graphs, workspaces
    # the vocoder's graph for this shape is captured on its second call: outside the timing
    mel = pkg("_dev").empty((len(groups[0]), 80, 2 * SWEEP_TOKENS))
    mel.fill_(-5.0)
    tts.hift.inference_batch(mel, use_graph=True)
    barrier()
    if full:
        prepared = [first] + [tts.prepare(sweep_requests(g, meta)) for g in groups[1:]]
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for pr in prepared:
            tts.run_prepared(pr, SWEEP_TOKENS)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        timed = len(prepared)
    else:
        ms = _timed(lambda: tts.run_prepared(first, SWEEP_TOKENS), 1)
        timed = 1
    barrier()
    ms = max_over_ranks(ms, world)
    sweep_s = ms * 1e-3 * (1 if full else batches)
    return {"workload": "config5 sweep: 256 utterances x 750 tokens (30 s), batches of 32 per GPU over %d GPU(s); "
                        "LM batch 32, CFG flow 2 x 32 at 1650 frames, vocoder 1500 frames decoded whole "
                        "(the time-chunked decode gives the same waveform up to rounding)" % world,
            "batches_per_gpu": batches, "batches_timed": timed, "batch_ms": ms / timed, "sweep_s": sweep_s,
            "value": SWEEP_UTTS / sweep_s, "unit": "30s-utterances/s",
            "lm_tok_s": SWEEP_UTTS * SWEEP_TOKENS / sweep_s, "extrapolated": not full}


def measure_strong(tts, meta, rank: int, world: int, reps: int, barrier):
    """Config 4 as a fixed job: 8 utterances in all, split over the ``world`` GPUs
    (1 per GPU at 8); the job's time is the slowest rank's."""
    per = max(UTTS // world, 1)
    mine = range(rank * per, min((rank + 1) * per, UTTS))
    prepared = tts.prepare(make_requests(mine, meta)) if len(mine) else None
    if prepared:
        tts.run_prepared(prepared, TOKENS)
        tts.run_prepared(prepared, TOKENS)          # the vocoder graph of this shape is captured here
    barrier()
    ms = _timed(lambda: tts.run_prepared(prepared, TOKENS), reps) if prepared else 0.0
    barrier()
    ms = max_over_ranks(ms, world)
    return {"workload": "config4 strong scaling: 8 utterances in all over %d GPU(s)" % world,
            "utterances": UTTS, "ms": ms, "value": UTTS / (ms * 1e-3), "unit": UNIT}



# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of the FF1 planes
# GEMM at the bench shape, from an ncu capture of `bench.py --kernel ff1q8p` (47,250,944 read,
# 38,543,360 written: part of the output planes is still in L2 when the kernel ends)
FF1_PLANES_DRAM_BYTES = 85_794_304


def ff1_planes_bytes(M: int, N: int, K: int) -> int:
    """Algorithmic bytes of one FF1 planes launch: A planes and exponents, the fp16 weights
    and fp32 transposed scales, the GELU output planes and exponents."""
    lde = -(-M // 16) * 16
    return M * 2 * K * 2 + (K // 64) * lde + N * K * 2 + (K // 64) * N * 4 + M * 2 * N * 2 + (N // 64) * lde


def dominant_kernel_roofline(tts, peaks):
    """Time the DiT FF1 GEMM at the bench shape in isolation (the largest kernel of the
    step) with CUDA events on its launching stream; achieved = 2*M*N*K / time.  In the
    balanced profile it is cv3_tc_gemm_q8_planes as the step runs it: int8 weights as
    stored, the activations as fp16 hi/lo planes (two fp16 MMAs per fp32 product), GELU
    written back as planes for FF2."""
    import torch
    L = pkg("_lib")
    dit = tts.flow.estimator
    dit.prepare()
    M = 2 * UTTS * 2 * (PROMPT_TOKENS + TOKENS)
    blk = dit.blocks[0].ff1
    q8 = type(blk).__name__ == "LinQ8"
    planes = q8 and dit.q8_planes
    st = torch.cuda.current_stream()
    x = torch.randn(M, blk.k, device="cuda")
    if planes:
        lde = (M + 15) // 16 * 16
        xp = torch.empty(M, 2 * blk.k, dtype=torch.float16, device="cuda")
        xe = torch.empty(blk.k // 64, lde, dtype=torch.int8, device="cuda")
        yp = torch.empty(M, 2 * blk.n, dtype=torch.float16, device="cuda")
        ye = torch.empty(blk.n // 64, lde, dtype=torch.int8, device="cuda")
        L.call("cv3_q8_split_rows", x.data_ptr(), blk.k, M, blk.k, xp.data_ptr(), xe.data_ptr(), lde, st.cuda_stream)

        def launch():
            blk.tc_planes(xp.data_ptr(), xe.data_ptr(), lde, M, None, 4, stream=st.cuda_stream,
                          out_planes=yp.data_ptr(), out_exps=ye.data_ptr(), out_lde=lde)
    else:
        y = torch.empty(M, blk.n, device="cuda")

        def launch():
            blk(x.data_ptr(), M, y.data_ptr(), stream=st.cuda_stream)
    for _ in range(3):
        launch()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 20
    torch.cuda.synchronize()
    e0.record(st)
    for _ in range(reps):
        launch()
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    flops = 2.0 * M * blk.n * blk.k
    achieved = flops / (ms * 1e-3) / 1e12
    peak = peaks.get("bf16_tflops")
    if planes:
        name = ("DiT ff1 GEMM (M=%d, N=%d, K=%d), int8 weights x activation planes (2 fp16 parts), "
                "GELU out as planes (cv3_tc_gemm_q8_planes mode 4)")
    elif q8:
        name = "DiT ff1 GEMM (M=%d, N=%d, K=%d), int8 weights x fp32 activations split in the GEMM (cv3_tc_gemm_q8)"
    else:
        name = "DiT ff1 GEMM (M=%d, N=%d, K=%d, fp32 via 3xTF32)"
    return {"kernel": name % (M, blk.n, blk.k), "bound": "tensor",
            "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak if peak else None,
            "peak_source": "measured bf16 dense (MEASURED_PEAKS.json, burst)",
            "avg_launch_ms": ms,
            "tensor_pipe": {"fp16_tflops_issued": (2.0 if q8 else 6.0) * achieved,
                            "frac_of_peak": (2.0 if q8 else 6.0) * achieved / peak if peak else None,
                            "note": "fp16/bf16-rate products issued per fp32 product: 2 (two fp16 parts of A "
                                    "against the exact fp16 weights)" if q8 else
                                    "3 tf32 products per fp32 product at half the bf16 rate"},
            "traffic": FF1_PLANES_DRAM_BYTES if planes else None, "traffic_unit": "bytes per launch",
            "algorithmic_bytes": ff1_planes_bytes(M, blk.n, blk.k) if planes else None}


def run_cuda(args, rank: int, world: int) -> None:
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
    synth, pipeline, L = pkg("synth"), pkg("pipeline"), pkg("_lib")
    W = synth.synthetic_weights("balanced")
    tts = pipeline.CosyVoice3CUDA(W)
    seeds = rank_seeds(rank)
    reqs = make_requests(seeds, W.meta)
    prepared = tts.prepare(reqs)
    for _ in range(max(args.warmup, 1)):
        wav, _ = tts.run_prepared(prepared, TOKENS)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    # -- value: inputs resident in HBM --------------------------------------------------
    barrier()
    torch.cuda.synchronize()
    l0 = L.executed_launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clk:
        e0.record()
        for _ in range(args.steps):
            wav, _ = tts.run_prepared(prepared, TOKENS)
        e1.record()
        torch.cuda.synchronize()
    barrier()
    launches = L.executed_launches() - l0
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)

    # -- e2e: host inputs in, host waveforms out, through the public API --------------------
    barrier()
    torch.cuda.synchronize()
    h2d = sum(int(np.asarray(r.text_ids).size + np.asarray(r.prompt_ids).size) * 8 +
              r.voice.speech_token.nbytes + r.voice.mel.nbytes + r.voice.embedding.nbytes for r in reqs)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(args.steps):
        wav_h, _ = tts.synthesize_greedy_batch(reqs, TOKENS, to_host=True)
    f1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1) / args.steps, world)
    d2h = int(wav_h.nbytes)

    peaks = json.load(open(PEAKS)) if os.path.exists(PEAKS) else {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0}
    roof = dominant_kernel_roofline(tts, peaks) if rank == 0 else None

    # -- the other configurations' numbers (every rank measures; rank 0 reports) -----------
    stages = {}
    if not args.no_stages:
        stages["config1_lm"] = measure_config1(tts, W.meta, peaks)
        Wf = synth.synthetic_weights("f32", stages=("flow", "hift"))
        stages["config2_flow"] = measure_config2(Wf, peaks)
        stages["config3_vocoder"] = measure_config3(Wf, peaks)
        del Wf
        stages["flow_hift_rtf"] = (stages["config2_flow"]["flow_s"] + stages["config3_vocoder"]["vocoder_s"]) / 10.0
        if world > 1:
            stages["config4_strong"] = measure_strong(tts, W.meta, rank, world, args.steps, barrier)
        stages["config5_sweep"] = measure_config5(tts, W.meta, rank, world, barrier)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_line(W, reqs[0])
    if rank == 0:
        total_utts = UTTS * world
        print(json.dumps({
            "metric": METRIC, "value": total_utts / (ms * 1e-3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_dict(args),
            "e2e": {"value": total_utts / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "roofline": roof,
            "cpu_baseline": cpu,
            "stages": stages,
        }), flush=True)


def run_sweep(args, rank: int, world: int) -> None:
    """``--sweep``: the whole config-5 sweep, one JSON line (rank 0)."""
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
    W = pkg("synth").synthetic_weights("balanced")
    tts = pkg("pipeline").CosyVoice3CUDA(W)
    barrier = (lambda: dist.barrier()) if world > 1 else (lambda: None)
    with ClockSampler(torch.cuda.current_device()) as clk:
        r = measure_config5(tts, W.meta, rank, world, barrier, full=True)
    if rank == 0:
        r.update({"n_gpus": world, "clocks": clk.summary(), "dtype": "f32", "data": "synthetic"})
        print(json.dumps(r), flush=True)


def run_slice(args) -> None:
    """Profiling slice: build everything, then, between cudaProfilerStart/Stop, run
    one eager batched LM decode step, one DiT forward at the bench's CFG shape and
    one batched vocoder pass (every kernel of a step, each launched once or per
    layer), for ``ncu --profile-from-start off``."""
    import torch
    synth, pipeline = pkg("synth"), pkg("pipeline")
    W = synth.synthetic_weights("balanced")
    tts = pipeline.CosyVoice3CUDA(W)
    reqs = make_requests(range(UTTS), W.meta)
    prepared = tts.prepare(reqs)
    tts.run_prepared(prepared, 4)                    # builds engines, graphs, tables
    eng = tts.llm.last_engine
    flow, dit = tts.flow, tts.flow.estimator
    N = 2 * (PROMPT_TOKENS + TOKENS)
    S = flow._solver(UTTS, N)
    mel = torch.randn(UTTS, 80, 2 * TOKENS, device="cuda")
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    st = torch.cuda.current_stream().cuda_stream
    eng.launches(st)
    pkg("_lib").call("cv3_dit_input_cat", S["x"].data_ptr(), S["cond"].data_ptr(), S["mu"].data_ptr(),
                     S["spk"].data_ptr(), UTTS, N, 80, 80, S["ws"].cat.data_ptr(), st)
    dit.modulation(S["tfeat"][0:1], S["mods"], S["temb"], st)
    dit.body(S["ws"], S["mods"], 0, st)
    tts.hift.inference_batch(mel)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print("slice done", flush=True)


def run_kernel(args) -> None:
    """One hot kernel alone at its bench shape, five launches (the small, self-contained
    case the ncu captures under profiles/ use): ``ff1`` the DiT FF GEMM, ``attention`` the
    DiT attention, ``conv`` the largest vocoder resblock conv, ``gemv`` the LM gate/up
    decode GEMV (batch 8)."""
    import math
    import numpy as np
    import torch
    L = pkg("_lib")
    common = pkg("models._common")
    st = torch.cuda.current_stream().cuda_stream
    torch.manual_seed(0)
    if args.kernel == "ff1":
        M, N, K = 2 * UTTS * 2 * (PROMPT_TOKENS + TOKENS), 2048, 1024
        a, b, c = torch.randn(M, K, device="cuda"), torch.randn(N, K, device="cuda") * 0.03, \
            torch.empty(M, N, device="cuda")
        lin = common.Lin(b)
        fn = lambda: lin.tc(a.data_ptr(), M, c.data_ptr(), 0, stream=st)
    elif args.kernel == "ff1q8":
        M, N, K = 2 * UTTS * 2 * (PROMPT_TOKENS + TOKENS), 2048, 1024
        quant = pkg("quant")
        w = (np.random.default_rng(0).normal(size=(N, K)) * 0.02).astype(np.float32)
        lin = common.LinQ8(quant.make_qtensor(w).to_device())
        a, c = torch.randn(M, K, device="cuda"), torch.empty(M, N, device="cuda")
        fn = lambda: lin(a.data_ptr(), M, c.data_ptr(), stream=st)
    elif args.kernel == "ff1q8p":
        # the same GEMM as the balanced DiT runs it: A as activation planes, GELU written
        # back as planes (mode 4)
        M, N, K = 2 * UTTS * 2 * (PROMPT_TOKENS + TOKENS), 2048, 1024
        quant = pkg("quant")
        w = (np.random.default_rng(0).normal(size=(N, K)) * 0.02).astype(np.float32)
        lin = common.LinQ8(quant.make_qtensor(w).to_device())
        a = torch.randn(M, K, device="cuda")
        lde = -(-M // 16) * 16
        pl = torch.empty((M, 2 * K), dtype=torch.float16, device="cuda")
        ex = torch.empty((K // 64, lde), dtype=torch.int8, device="cuda")
        op = torch.empty((M, 2 * N), dtype=torch.float16, device="cuda")
        oe = torch.empty((N // 64, lde), dtype=torch.int8, device="cuda")
        L.call("cv3_q8_split_rows", a.data_ptr(), K, M, K, pl.data_ptr(), ex.data_ptr(), lde, st)
        fn = lambda: lin.tc_planes(pl.data_ptr(), ex.data_ptr(), lde, M, None, 4, stream=st,
                                   out_planes=op.data_ptr(), out_exps=oe.data_ptr(), out_lde=lde)
    elif args.kernel == "attention":
        B, H, N, D = 2 * UTTS, 16, 2 * (PROMPT_TOKENS + TOKENS), 64
        qkv, o = torch.randn(B, N, 3 * H * D, device="cuda"), torch.empty(B, N, H * D, device="cuda")
        q = qkv.data_ptr()
        sb, sn = N * 3 * H * D, 3 * H * D
        fn = lambda: L.call("cv3_attention", q, sb, D, sn, q + H * D * 4, sb, D, sn, q + 2 * H * D * 4, sb, D, sn,
                            o.data_ptr(), N * H * D, D, H * D, B, H, H, N, N, D, 1.0 / math.sqrt(D), 0, 0, 0, st)
    elif args.kernel == "conv":
        C, T, k = 64, 120 * 2 * TOKENS, 7   # the 64-channel resolution: 120 samples per mel frame
        x, y = torch.randn(UTTS, C, T, device="cuda"), torch.empty(UTTS, C, T, device="cuda")
        cv = common.ConvTC((torch.randn(C, C, k, device="cuda") / math.sqrt(C * k)).half().float(),
                           torch.randn(C, device="cuda"))
        fn = lambda: cv(x, y, UTTS, T, T, dilation=3, pad_left=3 * (k - 1), stream=st)
    else:  # gemv
        quant = pkg("quant")
        w = (np.random.default_rng(0).normal(size=(9728, 896)) * 0.02).astype(np.float32)
        g = common.DecodeGemv(quant.make_qtensor(w).to_device(), None, torch.ones(896, device="cuda"), 1e-6,
                              swiglu=True)
        x, y = torch.randn(8, 896, device="cuda"), torch.empty(8, 4864, device="cuda")
        fn = lambda: g(x.data_ptr(), 8, y.data_ptr(), stream=st)
    for _ in range(5):
        fn()
    torch.cuda.synchronize()
    print("kernel %s: 5 launches done" % args.kernel, flush=True)
    if args.time:
        reps = 20
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        print(json.dumps({"kernel": args.kernel, "us_per_launch": round(e0.elapsed_time(e1) / reps * 1e3, 2)}),
              flush=True)


def trace_persistent(eng, B):
    """One 12-step persistent launch with step 8 traced (%globaltimer per CTA and phase):
    per phase kind (A qkv, B attention, C out-proj, D gate/up, E down, F head, G select),
    the mean over layers of the critical-path time (last CTA done minus the previous phase's
    last CTA done), the hand-over latency (first CTA past its wait minus the previous phase's
    last signal), the mean per-CTA work time and ring-slot wait."""
    import numpy as np
    import torch
    L = eng.c.num_hidden_layers
    nph = 5 * L + 2
    G = torch.cuda.get_device_properties(0).multi_processor_count
    tb = torch.zeros((G, nph, 6), dtype=torch.int64, device="cuda")
    P = eng._mk["params"]
    P.trace, P.trace_step = tb.data_ptr(), 8
    eng.steps_persistent(12)
    torch.cuda.synchronize()
    P.trace = None
    t = tb.cpu().numpy().astype(np.float64)
    names = ["A qkv", "B attention", "C out", "D gate/up", "E down"]
    out = {}
    done_prev = None
    rows = {}
    for ph in range(nph):
        kind = names[ph % 5] if ph < 5 * L else ("F head" if ph == nph - 2 else "G select")
        act = t[:, ph, 2] > 0
        if not act.any():
            continue
        done = t[act, ph, 2].max()
        started = t[act, ph, 1].min()
        r = rows.setdefault(kind, {"critical_us": [], "handover_us": [], "work_us": [], "ring_wait_us": [],
                                   "stage_us": [], "items_us": [], "signal_us": [], "ctas": int(act.sum())})
        if done_prev is not None:
            r["critical_us"].append((done - done_prev) / 1e3)
            r["handover_us"].append((started - done_prev) / 1e3)
        r["work_us"].append(float(np.mean(t[act, ph, 2] - t[act, ph, 1])) / 1e3)
        r["ring_wait_us"].append(float(np.mean(t[act, ph, 3])) / 1e3)
        st = act & (t[:, ph, 4] > 0)
        if st.any():
            r["stage_us"].append(float(np.mean(t[st, ph, 4] - t[st, ph, 1])) / 1e3)
            r["items_us"].append(float(np.mean(t[st, ph, 5] - t[st, ph, 4])) / 1e3)
        it = act & (t[:, ph, 5] > 0)
        if it.any():
            r["signal_us"].append(float(np.mean(t[it, ph, 2] - t[it, ph, 5])) / 1e3)
        done_prev = done
    for k, r in rows.items():
        out[k] = {kk: (round(float(np.mean(v)), 3) if isinstance(v, list) and v else v) for kk, v in r.items()}
    first = t[:, 0, 0][t[:, 0, 0] > 0].min() if (t[:, 0, 0] > 0).any() else 0
    last = t[:, nph - 1, 2].max()
    return {"trace_batch": B, "step_us": round((last - first) / 1e3, 1), "phases": out}


def run_lm_step(args) -> None:
    """Time the LM's graph-replayed decode step alone (full-size balanced LM, ``--lm-step B``
    sequences with 130-165-row prompts, caches of 512 positions; 20 warm-up steps, then 200
    steps between CUDA events on the replay stream); prints microseconds per step."""
    import numpy as np
    import torch
    B = args.lm_step
    W = pkg("synth").synthetic_weights("balanced", stages=("llm",))
    llm = pkg("models.llm")
    lm = llm.CosyVoice3LM(pkg("weights").DeviceWeights(W))
    rng = np.random.default_rng(3)
    prompts = [(rng.normal(size=(130 + 5 * i, 896)) * 0.1).astype(np.float32) for i in range(B)]
    if args.sampled:
        # the sampled step (device sampler as the last kernel), every sequence kept running
        # (all stop ids masked: strict min length over the whole timed run)
        cfg = llm.SamplingConfig(seed=0)
        eng = lm.sampling_engine(B, 512, 260, cfg, True)
        st = cfg.rng.bit_generator.state["state"]
        eng.run_sampled(prompts, [(st["state"], st["inc"])] * B, [2] * B, [2] * B)
        eng.min_len.fill_(250)
        eng.max_len.fill_(250)
        eng.done.zero_()
        eng.count.zero_()
    elif args.persistent:
        # the persistent kernel: 200 steps in one launch after a 20-step warm-up launch
        eng = lm.engine(B, 512, 260)
        eng.run(prompts, 21, persistent=True)
        torch.cuda.synchronize()
        if args.trace:
            print(json.dumps(trace_persistent(eng, B)), flush=True)
            return
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        eng.steps_persistent(200)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) / 200 * 1e3
        import ctypes
        code = ctypes.c_int(0)
        pkg("_lib").load().cv3_decode_status(ctypes.byref(code))
        print(json.dumps({"lm_decode_step_us": round(us, 1), "batch": B, "persistent": True, "status": code.value,
                          "weight_bytes_per_step": 375255804,
                          "weight_stream_gbs": round(375255804 / (us * 1e-6) / 1e9, 1)}), flush=True)
        return
    else:
        eng = lm.engine(B, 512, 260)
        eng.run(prompts, 2, use_graph=True)
    if not args.persistent:
        for _ in range(20):
            eng.step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 200
    e0.record()
    for _ in range(n):
        eng.step()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / n * 1e3
    if args.sampled:
        # the host-sampler path of generate(): a device forward, the log-probs to the host and
        # numpy's sampler, per token (batch 1)
        text = [int(W.meta.get("endofprompt_id", 151646))] + list(range(100, 130))
        cfg = llm.SamplingConfig(seed=0, min_token_text_ratio=0.0, max_token_text_ratio=2.0)
        t0 = time.perf_counter()
        ntok = len(list(lm.generate(text, (), [1, 2, 3], sampling=cfg, device_sampler=False)))
        host_ms = (time.perf_counter() - t0) * 1e3 / max(ntok, 1)
        print(json.dumps({"lm_sampled_step_us": round(us, 1), "batch": B,
                          "host_sampler_ms_per_token": round(host_ms, 3), "host_tokens": ntok}), flush=True)
        return
    print(json.dumps({"lm_decode_step_us": round(us, 1), "batch": B, "weight_bytes_per_step": 375255804,
                      "weight_stream_gbs": round(375255804 / (us * 1e-6) / 1e9, 1)}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--lm-step", type=int, default=0, metavar="B",
                    help="time the LM decode step alone at batch B (1..32)")
    ap.add_argument("--persistent", action="store_true",
                    help="with --lm-step: the persistent decode kernel (every step in one launch)")
    ap.add_argument("--trace", action="store_true",
                    help="with --lm-step B --persistent: per-phase timestamps of one step")
    ap.add_argument("--sampled", action="store_true",
                    help="with --lm-step: the sampled step (device sampler) and the host-sampler path")
    ap.add_argument("--slice", action="store_true", help="profiling slice (see run_slice)")
    ap.add_argument("--kernel", choices=["ff1", "ff1q8", "ff1q8p", "attention", "conv", "gemv"],
                    help="run one hot kernel alone at its bench shape (for ncu captures)")
    ap.add_argument("--time", action="store_true",
                    help="with --kernel: also time 20 more launches (CUDA events on the launching stream)")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["cuda", "reference"], default="cuda")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-full-utterance", action="store_true",
                    help="reference arm: skip the one complete (unextrapolated) CPU utterance")
    ap.add_argument("--no-stages", action="store_true", help="skip the config 1-3 and 5 stage numbers")
    ap.add_argument("--sweep", action="store_true",
                    help="config 5 alone: all 256 utterances, sharded over the ranks, every batch timed")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    if world > 1 and args.impl == "cuda":
        import datetime
        import torch.distributed as dist
        import torch
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        local = int(os.environ.get("LOCAL_RANK", 0))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    try:
        if args.lm_step:
            run_lm_step(args)
        elif args.kernel:
            run_kernel(args)
        elif args.slice:
            run_slice(args)
        elif args.impl == "reference":
            run_reference(args, rank, world)
        elif args.sweep:
            run_sweep(args, rank, world)
        else:
            run_cuda(args, rank, world)
    finally:
        if world > 1 and args.impl == "cuda":
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

/*
 * cv3cuda -- the C ABI of the B200 (sm_100a) kernel layer for CosyVoice 3.
 *
 * Each entry point replaces one operation of the reference's NumPy kernel
 * layer (cv3cpu/ops.py, cv3cpu/quant.py, cv3cpu/torch_rng.py) or one fused
 * group of them used by a model stage (cv3cpu/models/*.py).  The comment on
 * every declaration names the reference function (path:line) it replaces.
 *
 * Conventions
 *   - Plain pointers and sizes only.  Unless a parameter says "host", every
 *     pointer is a CUDA device pointer on the current device.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default).
 *     Calls are asynchronous and stream-ordered; none allocates device memory
 *     unless its comment says so, and none synchronises the stream.
 *   - Every call returns a status: CV3_OK (0) or one of the CV3_ERR_* codes.
 *     cv3_last_error() returns a message for the last failure on the calling
 *     host thread.  The Python host maps CV3_ERR_VALUE to ValueError,
 *     CV3_ERR_INDEX to IndexError and the rest to RuntimeError, the
 *     exception types the reference raises for the same conditions.
 *   - float tensors are row-major, contiguous unless a leading dimension
 *     (ld*) is given.  q8 weights use the "balanced" layout: int8 q[N][Kp],
 *     Kp = K rounded up to 64, and float16 scales s[N][Kp/64] (passed as
 *     uint16_t bit patterns); W[n][k] = float(q[n][k]) * float(s[n][k/64]).
 */
#ifndef CV3CUDA_H
#define CV3CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CV3_OK 0
#define CV3_ERR_VALUE 1       /* bad shape / argument  -> ValueError   */
#define CV3_ERR_INDEX 2       /* id outside a table    -> IndexError   */
#define CV3_ERR_CUDA 3        /* CUDA runtime failure  -> RuntimeError */
#define CV3_ERR_UNSUPPORTED 4 /* configuration not built -> RuntimeError */

#define CV3_ABI_VERSION 1

/* ------------------------------------------------------------------ */
/* library                                                             */
/* ------------------------------------------------------------------ */

/* Message of the last failed call on this host thread ("" if none). */
const char* cv3_last_error(void);

/* CV3_ABI_VERSION of the loaded library. */
int cv3_abi_version(void);


/* Kernels this library has launched (or recorded into a graph being
 * captured) since it was loaded, over all host threads. */
unsigned long long cv3_launch_count(void);

/* SM count and compute capability of the current device. */
int cv3_device_info(int* sm_count, int* cc_major, int* cc_minor);

/* Device memory and copies for a host without a GPU framework (the NumPy +
 * ctypes host of the ops layer, which replaces cv3cpu/ops.py's NumPy arrays by
 * device arrays made here): cudaMalloc / cudaFree of `bytes` (0: *ptr = NULL),
 * one cudaMemcpyAsync per call (kind 0 host->device, 1 device->host, 2
 * device->device; pageable host memory makes the copy return once the host side
 * may be reused), cudaMemsetAsync, cudaStreamSynchronize, cudaMemGetInfo.  No
 * counterpart in the reference (NumPy owns its memory there). */
int cv3_device_alloc(int64_t bytes, void** ptr);
int cv3_device_free(void* ptr);
int cv3_memcpy(void* dst, const void* src, int64_t bytes, int kind, void* stream);
int cv3_memset(void* dst, int value, int64_t bytes, void* stream);
int cv3_stream_synchronize(void* stream);
int cv3_mem_get_info(int64_t* free_bytes, int64_t* total_bytes);

/* ------------------------------------------------------------------ */
/* linear layers                                                        */
/* ------------------------------------------------------------------ */

/* y[m][n] = sum_k x[m][k] * W[n][k] + bias[n] (+ residual[m][n]) for a q8 W.
 * Replaces cv3cpu/quant.py:156-204 (qmatmul with a QTensor, reached through
 * cv3cpu/ops.py:121 linear).  x: [m][k] fp32 with row stride ldx; bias and
 * residual may be NULL; y: [m][n] with row stride ldy (y may alias residual).
 * Any m >= 1; the weight stream is read once for up to 8 rows per pass. */
int cv3_q8_linear(const float* x, int64_t m, int64_t k, int64_t ldx,
                  const int8_t* q, const uint16_t* scales, int64_t n, int64_t kp,
                  const float* bias, const float* residual,
                  float* y, int64_t ldy, void* stream);

/* Decode-step q8 GEMV for 1..8 activation rows with the Qwen2 layer's
 * fusions: y = epi(norm(x) . W^T + bias) where norm is RMSNorm with weight
 * norm_w (NULL: none; cv3cpu/ops.py:101-104), epi adds residual (y may alias
 * it) or, with swiglu = 1 and weight rows interleaved gate/up, writes
 * y[m][i] = silu(row 2i) * row 2i+1 (qwen2.py:175-177).  `splits` > 1 splits K
 * over CTAs: then workspace must hold splits*8*n floats and counters n/32 ints,
 * zero on the first call and left zero by every call (per-weight buffers; do
 * not share them between concurrent calls).  Replaces the per-token
 * ops.linear calls of qwen2.py:156-177 and llm.py:74-78. */
int cv3_q8_decode_gemv(const float* x, int64_t m, int64_t k, int64_t ldx, const int8_t* q,
                       const uint16_t* scales, int64_t n, int64_t kp, const float* bias,
                       const float* residual, const float* norm_w, float eps, int swiglu, float* y,
                       int64_t ldy, int64_t splits, float* workspace, int64_t workspace_floats,
                       int* counters, void* stream);

/* cv3_q8_decode_gemv on the tensor cores (warp MMA m16n8k16: int8 weights are
 * exact bf16, the activations enter as three exact bf16 parts, the fp16 group
 * scale multiplies each 64-wide group's fp32 partial sum), for 1..32 activation
 * rows (the batch-32 decode of config 5; a row's result does not depend on m).
 * Same operands, fusions and output as cv3_q8_decode_gemv; needs K a multiple
 * of 64 with no padding (kp == k), K <= 5120, 16-byte aligned x rows; a CTA
 * stages its rows' K range in shared memory, so m > 8 with a long K needs
 * `splits` (CV3_ERR_VALUE otherwise).  `splits` > 1 spreads K over that many
 * CTAs per row tile with a deterministic reduction (a cluster for up to 8
 * splits; with a fused RMSNorm at most 8, the cluster's first CTA adding the
 * others' sums of squares); more than 8 splits need workspace >= splits*n*8*B floats
 * (B = 1 for m <= 8, 2 for m <= 16, else 4) and counters (one per 16-row tile,
 * or 32-row when n >= 4096 and a CTA takes at most 16 scale groups) zeroed
 * once, left zeroed.  Replaces the per-token ops.linear calls of
 * qwen2.py:156-177 and llm.py:74-78 (quant.py:156-204 with m <= 32). */
int cv3_q8_decode_gemv_mma(const float* x, int64_t m, int64_t k, int64_t ldx, const int8_t* q,
                           const uint16_t* scales, int64_t n, int64_t kp, const float* bias, const float* residual,
                           const float* norm_w, float eps, int swiglu, float* y, int64_t ldy, int64_t splits,
                           float* workspace, int64_t workspace_floats, int* counters, void* stream);

/* Error word of cv3_q8_decode_gemv_mma, read and cleared: 0, or 1 when a CTA's
 * bulk copy of the activation rows did not land within 2 s (that CTA then wrote
 * nothing).  No counterpart in the reference (a device-side wait bound). */
int cv3_decode_gemv_status(int* code);

/* Same contract for an fp32 weight W[n][k] (row stride ldw); replaces the
 * plain-array branch of cv3cpu/quant.py:165-170. fp32-exact SIMT math. */
int cv3_f32_linear(const float* x, int64_t m, int64_t k, int64_t ldx,
                   const float* w, int64_t n, int64_t ldw,
                   const float* bias, const float* residual,
                   float* y, int64_t ldy, void* stream);

/* Dequantise q8 rows [0, n) into fp32 out[n][k] (k <= kp, padding dropped).
 * Replaces cv3cpu/quant.py:110-133 (QTensor.dequant_rows). */
int cv3_q8_dequant(const int8_t* q, const uint16_t* scales, int64_t n, int64_t kp,
                   int64_t k, float* out, void* stream);

/* The q4 "tiny"-profile linear, cv3cpu/quant.py:156-204 with a QTensor of kind
 * "q4" (format quant.py:70-86, expansion :124-131): y[m][n] = x[m][k] . W[n][k]
 * (+ bias[n]) (+ residual[m][n]), W = (code - 8) * fp16 scale per 32-wide block;
 * payload uint8 [n][kp/2] (byte j of a block: code j low nibble, code j + 16 high
 * nibble), scales [n][kp/32], kp = k rounded up to 32.  Any m (8 rows per pass). */
int cv3_q4_linear(const float* x, int64_t m, int64_t k, int64_t ldx, const uint8_t* q, const uint16_t* scales,
                  int64_t n, int64_t kp, const float* bias, const float* residual, float* y, int64_t ldy,
                  void* stream);

/* q4 weight -> fp32 [n][k] (exact); cv3cpu/quant.py:110-133 (QTensor.dequant_rows, q4 branch). */
int cv3_q4_dequant(const uint8_t* q, const uint16_t* scales, int64_t n, int64_t kp, int64_t k, float* out,
                   void* stream);

/* ------------------------------------------------------------------ */
/* elementwise and normalisation                                        */
/* ------------------------------------------------------------------ */

#define CV3_ACT_SILU 0       /* cv3cpu/ops.py:30  */
#define CV3_ACT_SIGMOID 1    /* cv3cpu/ops.py:34  */
#define CV3_ACT_GELU_TANH 2  /* cv3cpu/ops.py:41  */
#define CV3_ACT_GELU_ERF 3   /* cv3cpu/ops.py:46  (A&S 7.1.26 erf) */
#define CV3_ACT_MISH 4       /* cv3cpu/ops.py:63  */
#define CV3_ACT_ELU 5        /* cv3cpu/ops.py:69  (param = alpha) */
#define CV3_ACT_LEAKY_RELU 6 /* cv3cpu/ops.py:73  (param = slope) */
#define CV3_ACT_TANH 7       /* np.tanh, cv3cpu/models/hift.py:111 */
#define CV3_ACT_EXP 8        /* np.exp */

/* y[i] = act(x[i]) for i < n (y may alias x). */
int cv3_unary(int act, float param, const float* x, int64_t n, float* y, void* stream);

/* y = rms_norm(x, w, eps) over rows of length dim; cv3cpu/ops.py:101-104. */
int cv3_rms_norm(const float* x, const float* w, int64_t rows, int64_t dim, float eps,
                 float* y, void* stream);

/* y = layer_norm(x, w, b, eps) over rows; w, b may be NULL; cv3cpu/ops.py:107-118. */
int cv3_layer_norm(const float* x, const float* w, const float* b, int64_t rows,
                   int64_t dim, float eps, float* y, void* stream);

/* Row-wise softmax (log=0) or log_softmax (log=1); cv3cpu/ops.py:84-93. */
int cv3_softmax(const float* x, int64_t rows, int64_t dim, int log, float* y, void* stream);

/* Snake over [batch][C][T]: y = x + sin(a x)^2 / (a + 1e-9), a per channel;
 * cv3cpu/ops.py:77-81. */
int cv3_snake(const float* x, const float* alpha, int64_t batch, int64_t channels, int64_t t,
              float* y, void* stream);


/* ------------------------------------------------------------------ */
/* gathers, convolution, attention                                      */
/* ------------------------------------------------------------------ */

#define CV3_TABLE_F32 0
#define CV3_TABLE_F16 1
#define CV3_TABLE_Q8 2
#define CV3_TABLE_Q4 3

/* out[i][:] = table[ids[i]][:] widened to fp32 (q8 / q4: dequantised row).
 * Replaces cv3cpu/ops.py:126-144 (embedding).  ids: device int64[n];
 * table: f32/f16 [rows][dim], q8 [rows][kp] or q4 [rows][kp/2] with scales.  Rows outside
 * the table produce zeros and increment *bad (device int, may be NULL);
 * the host raises IndexError before launching for host-side ids. */
int cv3_embedding(const void* table, int kind, const uint16_t* scales, int64_t rows, int64_t dim,
                  int64_t kp, const int64_t* ids, int64_t n, float* out, int64_t ldo, int* bad,
                  void* stream);

/* Batched 1-D cross-correlation: x [batch][cin][t_in] -> y [batch][cout][t_out]
 * with weight [cout][cin/groups][k], optional bias, zero padding
 * (pad_left, pad_right), stride, dilation, groups.  t_out must equal
 * (t_in + pad_left + pad_right - dilation*(k-1) - 1)/stride + 1.
 * Replaces cv3cpu/ops.py:165-219 (conv1d) and :222-236 (depthwise_conv1d). */
int cv3_conv1d(const float* x, int64_t batch, int64_t cin, int64_t t_in, const float* w, int64_t cout,
               int64_t k, int64_t stride, int64_t dilation, int64_t groups, int64_t pad_left,
               int64_t pad_right, const float* bias, float* y, int64_t t_out, void* stream);

#define CV3_MASK_NONE 0
#define CV3_MASK_CAUSAL 1 /* key j visible to query i iff j <= i + a          */
#define CV3_MASK_CHUNK 2  /* chunk size a, b chunks of left context (-1: all) */

/* Exact-softmax attention.  Element (b, h, i, d) of q/k/v/o lives at
 * base + b*s_b + h*s_h + i*s_n + d (strides in floats), so (H, N, D) and
 * token-major (B, N, H*D) layouts are both read in place.  GQA: query head h
 * uses kv head h / (heads / kv_heads).  Replaces cv3cpu/ops.py:267-310 (sdpa
 * with _block_mask :244-264); head_dim <= 64.  Head dim 64 with 16-byte
 * aligned rows (the DiT and Qwen2 shapes) and more than 4 queries runs on the
 * tensor cores (tcgen05, 3xTF32, flash tiling); other shapes on CUDA cores. */
int cv3_attention(const float* q, int64_t qsb, int64_t qsh, int64_t qsn,
                  const float* k, int64_t ksb, int64_t ksh, int64_t ksn,
                  const float* v, int64_t vsb, int64_t vsh, int64_t vsn,
                  float* o, int64_t osb, int64_t osh, int64_t osn,
                  int64_t batch, int64_t heads, int64_t kv_heads, int64_t n, int64_t m, int64_t d,
                  float scale, int mask_kind, int64_t mask_a, int64_t mask_b, void* stream);

/* ------------------------------------------------------------------ */
/* spectral and resampling                                               */
/* ------------------------------------------------------------------ */

/* One-sided STFT of batch signals x [batch][len], reflect-padded by n_fft/2,
 * window win[n_fft]; out [batch][2F][frames], F = n_fft/2+1, rows [0,F) real
 * and [F,2F) imaginary parts.  frames = 1 + len/hop (centre padding).
 * Replaces cv3cpu/ops.py:346-355 (stft) as the vocoder consumes it
 * (cv3cpu/models/hift.py:198-199). */
int cv3_stft(const float* x, int64_t batch, int64_t len, int64_t n_fft, int64_t hop, const float* win,
             float* out, int64_t frames, void* stream);

#define CV3_ISTFT_REIM 0 /* spec rows: [0,F) real, [F,2F) imaginary                 */
#define CV3_ISTFT_HIFT 1 /* spec rows: log-magnitude, phase angle (hift.py:204-208) */

/* Inverse STFT with window-square normalisation and clip to +-limit.
 * y[b][t] = overlap-add sample (t + offset), t < out_len; offset = n_fft/2
 * gives the centred signal.  frame_scratch: device float [batch][frames][n_fft].
 * Replaces cv3cpu/ops.py:358-377 (istft) and cv3cpu/models/hift.py:204-210. */
int cv3_istft(const float* spec, int mode, int64_t batch, int64_t frames, int64_t n_fft, int64_t hop,
              const float* win, float limit, int64_t offset, float* frame_scratch, float* y,
              int64_t out_len, void* stream);

/* cv3_istft without any device allocation, for callers that cannot allocate
 * when they run the vocoder's inverse STFT (a real-time audio callback must
 * not block on cudaMalloc; a host whose memory pool already owns the GPU has
 * nothing left to allocate).  No counterpart in the reference (its NumPy iSTFT
 * allocates freely); same arguments and results as cv3_istft minus
 * frame_scratch.  The frame buffer is a 4 MiB array built into the library
 * (batch * frames * n_fft <= 1,048,576 floats, CV3_ERR_VALUE beyond), held by
 * every device that loads the library until exit and shared by all calls:
 * calls whose kernels may overlap on the GPU race and must be ordered by the
 * caller.  The first call on each device looks up the array's device address;
 * make that call before any stream capture (a first call on a capturing stream
 * returns CV3_ERR_VALUE and does nothing). */
int cv3_istft_noalloc(const float* spec, int mode, int64_t batch, int64_t frames, int64_t n_fft, int64_t hop,
                      const float* win, float limit, int64_t offset, float* y, int64_t out_len, void* stream);

/* y [rows][t*scale] = x repeated along time; cv3cpu/ops.py:335-336. */
int cv3_interpolate_nearest(const float* x, int64_t rows, int64_t t, int64_t scale, float* y, void* stream);

/* y [rows][size] = x[:, i0] * (1 - w) + x[:, i1] * w with host-built index/weight
 * tables (device int64 i0, i1, float w); cv3cpu/ops.py:318-332. */
int cv3_interpolate_linear(const float* x, int64_t rows, int64_t t, const int64_t* i0, const int64_t* i1,
                           const float* w, int64_t size, float* y, void* stream);

/* ------------------------------------------------------------------ */
/* torch CPU generator replica                                          */
/* ------------------------------------------------------------------ */

/* out[i] = float32 uniform number (skip + i) of torch.manual_seed(seed)'s
 * stream (MT19937, low 24 bits); torch_rng.py:88-91 and :145-150. */
int cv3_torch_rand(uint64_t seed, int64_t skip, int64_t n, float* out, void* stream);

/* Raw tempered MT19937 words of torch's CPU generator seeded with `seed`, starting `skip`
 * words into the stream: TorchMT19937.next_u32 (cv3cpu/torch_rng.py:71-86). */
int cv3_torch_u32(uint64_t seed, int64_t skip, int64_t n, uint32_t* out, void* stream);

/* n double uniforms from consecutive word pairs (first word high, 53 bits), starting `skip`
 * words in: TorchMT19937.random_float64 (cv3cpu/torch_rng.py:93-102); consumes 2n words. */
int cv3_torch_rand64(uint64_t seed, int64_t skip, int64_t n, double* out, void* stream);

/* out[0..n) = torch.randn(n) drawn from torch.manual_seed(seed)'s generator
 * after `skip` 32-bit words were consumed (skip = 0: a fresh seed), bit-exact
 * with cv3cpu/torch_rng.py:117-142.  Consumes n (+16 when n % 16 != 0) words,
 * or 4*ceil(n/2) words when n < 16.  scratch: 128 device bytes. */
int cv3_torch_randn(uint64_t seed, int64_t skip, int64_t n, float* out, void* scratch, void* stream);

/* ------------------------------------------------------------------ */
/* Qwen2 decode step (cv3cpu/models/qwen2.py:139-179, llm.py:112-121)    */
/* ------------------------------------------------------------------ */

/* RoPE + KV append for `rows` rows of fused qkv [rows][ldq] (q heads, then k,
 * then v, head_dim each).  Row r belongs to sequence seq[r] at position pos[r]
 * (device int32).  q is rotated into q_out [rows][heads][head_dim]; k is
 * rotated and v copied into k_cache/v_cache [seq][kv_heads][cap][head_dim].
 * Half-split rotation x*cos + rotate_half(x)*sin with host-built float64->
 * float32 tables [positions][head_dim]; replaces qwen2.py:64-71 apply_rope and
 * :108-118 KVCache.append. */
int cv3_rope_qkv_append(const float* qkv, int64_t rows, int64_t ldq, const float* cos_table,
                        const float* sin_table, const int* seq, const int* pos, int64_t heads,
                        int64_t kv_heads, int64_t head_dim, float* q_out, float* k_cache, float* v_cache,
                        int64_t cap, void* stream);

/* One-query-per-sequence attention over the cache: out [batch][heads*head_dim]
 * from q [batch][heads][head_dim] and the first lens[b] (device int32) cached
 * keys of sequence b.  Replaces ops.sdpa with mask None for a 1-token step
 * (qwen2.py:148, :169). */
int cv3_decode_attention(const float* q, const float* k_cache, const float* v_cache, const int* lens,
                         int64_t batch, int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t cap,
                         float scale, float* out, void* stream);

/* One decode step's RoPE, KV-cache append and attention in one launch: qkv rows b
 * (sequence b, ldq floats apart) hold the q/k/v projection ((heads + 2 kv_heads)
 * heads of 64); each (sequence, kv head) rotates its query heads and its key at
 * pos[b] (half-split RoPE with the [position][64] cos / sin tables, rounded as
 * cv3_rope_qkv_append), appends key and value at pos[b] (not stored outside
 * [0, cap)), then attends like cv3_decode_attention over lens[b] cached rows.
 * Same results as cv3_rope_qkv_append followed by cv3_decode_attention, up to the
 * order of a score's sums.  The cached rows below pos[b] are copied into shared
 * memory before the launch's dependency wait, so pos[b] and those rows must have
 * been written at least two launches earlier on the stream (the decode chain
 * writes them one step earlier); a position that changed by the wait falls back
 * to global reads. */
/* Error word of cv3_decode_rope_attention, read and cleared: 0, or 1 when a CTA's
 * staged key/value copy did not land within 2 s (that CTA then wrote nothing).
 * No counterpart in the reference (a device-side wait bound). */
int cv3_decode_attention_status(int* code);

int cv3_decode_rope_attention(const float* qkv, int64_t ldq, const float* cos_table, const float* sin_table,
                              const int* pos, float* k_cache, float* v_cache, const int* lens, int64_t batch,
                              int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t cap, float scale, float* out,
                              void* stream);

/* One sampled decode step per sequence, replacing the host sampler of
 * cv3cpu/models/llm.py:107-123 (generate), :125-149 (_sample) and :37-49
 * (nucleus_sampling): logits [batch][vocab] -> log_softmax -> stop ids
 * [speech_token_size, +200) masked while count[b] < min_len[b] (only the first
 * unless strict_min_len) -> softmax -> the top_k (<= 32) most probable in stable
 * order, kept while their float64 running sum is below top_p -> a draw from them
 * -> if that token occurs >= win_size * tau_r times in the last win_size tokens
 * of history, a redraw from the full distribution without it.  rng_state
 * [batch][4] holds numpy PCG64 states (state hi, lo, increment hi, lo) and is
 * advanced exactly as numpy's Generator.choice advances it.  A stop id sets
 * done[b] (nothing recorded); otherwise the token goes to history[b][count[b]],
 * next_ids[b], count/pos/lens advance, and done[b] is set once count reaches
 * max_len[b].  Sequences with done[b] set are left untouched.  logp_out
 * (optional) receives the log-probabilities. */
int cv3_sample_select(const float* logits, int64_t batch, int64_t vocab, int64_t speech_token_size,
                      const int* min_len, const int* max_len, int strict_min_len, double top_p, int64_t top_k,
                      int64_t win_size, double tau_r, uint64_t* rng_state, int64_t* next_ids, int* pos, int* lens,
                      int64_t* history, int64_t hist_stride, int* count, int* done, float* logp_out,
                      void* stream);

/* y[r][i] = silu(gu[r][i]) * gu[r][inter + i]; qwen2.py:175-177. */
int cv3_swiglu(const float* gate_up, int64_t rows, int64_t inter, float* y, void* stream);

/* Greedy head for `batch` rows of logits [batch][vocab]: log_softmax over the
 * vocabulary (llm.py:114; stored to logp_out when non-NULL), token = first
 * argmax of the log-probabilities over [0, select) (stop ids masked), written
 * to next_ids[b] and history[b][*step]; then pos[b]++, lens[b]++ and, when
 * step is non-NULL, ++*step.  All state is device memory. */
int cv3_head_select(const float* logits, int64_t batch, int64_t vocab, int64_t select, float* logp_out,
                    int64_t* next_ids, int* pos, int* lens, int64_t* history, int64_t hist_stride,
                    int* step, void* stream);

/* ------------------------------------------------------------------ */
/* DiT flow estimator and Euler/CFG solve (cv3cpu/models/dit.py, flow.py) */
/* ------------------------------------------------------------------ */

/* CFG input rows: out [2*utts][frames][3*mel + spk_dim] = concat(x, cond, mu,
 * spk) for b = 2u (utterance u) and concat(x, 0, 0, 0) for b = 2u+1; x, cond,
 * mu are channel-major [utts][mel][frames], spk [utts][spk_dim].
 * Replaces dit.py:92-97 with flow.py:71-77. */
int cv3_dit_input_cat(const float* x, const float* cond, const float* mu, const float* spk, int64_t utts,
                      int64_t frames, int64_t mel, int64_t spk_dim, float* out, void* stream);

/* y = layer_norm(h, eps) * (1 + scale) + shift per row (no affine); row r
 * uses scale/shift + (r / rows_per_group) * mod_stride (rows_per_group 0:
 * one shared vector).  Replaces dit.py:168-169, :171-172, :178. */
int cv3_ln_modulate(const float* h, int64_t rows, int64_t dim, float eps, const float* scale,
                    const float* shift, int64_t rows_per_group, int64_t mod_stride, float* y, void* stream);

/* h += gate * y per row (gate chosen like cv3_ln_modulate); dit.py:170, :173. */
int cv3_gate_residual(float* h, const float* y, const float* gate, int64_t rows, int64_t dim,
                      int64_t rows_per_group, int64_t gate_stride, void* stream);

/* In place, on rows of fused qkv [rows][ld]: rotate channel pairs
 * (2i, 2i+1), i < width/2, of q (offset 0) and k (offset k_offset) by the
 * angle tables [frames][width] at position row % frames -- the reference's
 * rotate-before-head-split quirk that only moves head 0 (dit.py:32-54). */
int cv3_partial_rope(float* qkv, int64_t rows, int64_t ld, int64_t k_offset, int64_t frames,
                     int64_t width, const float* cos_table, const float* sin_table, void* stream);

/* out[b] = in[b]^T for batch matrices [rows][cols]; accumulate=1 adds. */
int cv3_transpose(const float* in, int64_t batch, int64_t rows, int64_t cols, float* out, int accumulate,
                  void* stream);

/* Euler step with guidance: x[u][c][n] += dt * ((1 + cfg) * d[2u][n][c] - cfg * d[2u+1][n][c]),
 * d token-major [2*utts][frames][mel]; flow.py:86-87. */
int cv3_cfg_euler(float* x, const float* d, int64_t utts, int64_t mel, int64_t frames, double cfg_rate,
                  float dt, void* stream);

/* y = x / max(||x||_2, 1e-12) per row; flow.py:105-106. */
int cv3_l2_normalize(const float* x, int64_t rows, int64_t dim, float* y, void* stream);

/* ------------------------------------------------------------------ */
/* HiFT vocoder (cv3cpu/models/hift.py)                                 */
/* ------------------------------------------------------------------ */

/* f0[b][t] = float32(|sum_c double(x[b][c][t]) * w[c] + b[0]|): the F0 head's
 * float64 classifier over float32 condnet features; hift.py:69-72, :217. */
int cv3_f0_classifier(const float* x, int64_t batch, int64_t channels, int64_t t, const double* w,
                      const double* b, float* f0, void* stream);

/* NSF harmonic source: out[b][s], s < up*t, = tanh(sum_h sw[s][h] * w[h] + bias)
 * with sw = float32(sin(phase[t][h])) * alpha * uv + amp * noise[s][h],
 * phase = cumsum_t((f0*(h+1)/sample_rate) mod 1) * 2pi * up in float64,
 * uv = f0 > voiced_threshold, amp = uv*sigma + (1-uv)*alpha/3.  noise is the
 * fixed uniform dither [up*t][harmonics]; sines_scratch holds
 * [batch][t][harmonics] floats.  Replaces hift.py:90-111. */
int cv3_nsf_source(const float* f0, int64_t batch, int64_t t, int64_t harmonics, int64_t sample_rate,
                   int64_t up, double alpha, double sigma, double voiced_threshold, const float* noise,
                   const float* w, const float* bias, float* sines_scratch, float* out, void* stream);

#define CV3_BIN_ADD 0
#define CV3_BIN_SUB 1
#define CV3_BIN_MUL 2
#define CV3_BIN_DIV_SCALAR 3
#define CV3_BIN_MUL_SCALAR 4

/* y = a (op) b, or a (op) scalar; the residual sums and the resblock mean of
 * hift.py:128, :164-165. */
int cv3_binary(int op, const float* a, const float* b, float scalar, int64_t n, float* y, void* stream);

/* y[r] = [x[r][1], x[r][0..t)]: ReflectionPad1d((1, 0)); hift.py:144. */
int cv3_reflect_left1(const float* x, int64_t rows, int64_t t, float* y, void* stream);

/* ------------------------------------------------------------------ */
/* tensor-core fp32 GEMM (tcgen05 + TMEM + TMA, 3xTF32)                 */
/* ------------------------------------------------------------------ */

#define CV3_EPI_BIAS 0          /* c = acc + bias                              */
#define CV3_EPI_BIAS_GELU 1     /* c = gelu_tanh(acc + bias)                   */
#define CV3_EPI_GATED_RESIDUAL 2 /* c += gate[row/rows_per_group] * (acc + bias) */
#define CV3_EPI_RESIDUAL 3      /* c += acc + bias                             */

/* c[m][n] = epilogue(sum_k a[m][k] * b[n][k]) with fp32 operands computed as
 * 3xTF32 on the tensor cores (hi*hi + hi*lo + lo*hi, fp32 accumulation in
 * TMEM): the fp32 linears of the DiT (cv3cpu/ops.py:121 via quant.py:165-170
 * for plain weights), with the bias / GELU-tanh (dit.py:140) / gated
 * residual (dit.py:170, :173) epilogues fused.  k % 4 == 0, 16-byte aligned
 * rows; bias may be NULL. */
int cv3_tc_gemm(const float* a, int64_t lda, const float* b, int64_t ldb, float* c, int64_t ldc, int64_t m,
                int64_t n, int64_t k, int mode, const float* bias, const float* gate, int64_t rows_per_group,
                int64_t gate_stride, void* stream);

/* lo[i] = x[i] - tf32(x[i]) (x with its low 13 mantissa bits cleared): the
 * exact remainder the 3xTF32 products need.  Made once per weight matrix. */
int cv3_tf32_lo(const float* x, int64_t n, float* lo, void* stream);

/* The DiT's GEMM: cv3_tc_gemm's contract (same operand rules -- k % 4 == 0,
 * 16-byte aligned rows --, epilogue modes and 3xTF32 accuracy) with B given as
 * its fp32 values plus the remainders of cv3_tf32_lo (same ldb), on persistent
 * CTAs that split A on the fly, spread the products over four TMEM
 * accumulators (hi*hi of even and of odd K blocks, lo*hi, hi*lo) and overlap
 * each tile's epilogue with the next tile's MMAs. */
int cv3_tc_gemm_split(const float* a, int64_t lda, const float* b, const float* b_lo, int64_t ldb, float* c,
                      int64_t ldc, int64_t m, int64_t n, int64_t k, int mode, const float* bias, const float* gate,
                      int64_t rows_per_group, int64_t gate_stride, void* stream);

/* The balanced profile's q8 linears on the tensor cores with the int8 weights as
 * they are stored (replaces cv3cpu/quant.py:156-204 qmatmul on the DiT's block
 * matrices, cv3cpu/models/dit.py:114-142):
 *   C = epilogue( sum_g s[n][g] * (A[:, 64g..64g+63] . q[n][64g..64g+63]) )
 * A fp32 [m][lda] (16-byte aligned rows), each 64-wide K group of a row split into
 * two fp16 parts after a power-of-two scaling (22 significant bits, the precision
 * of the 3xTF32 split); w16 = q as fp16 [n][k] and scales_t = s as fp32 [k/64][n],
 * both made once by cv3_q8_gemm_prepare.  n % 128 == 0, k % 64 == 0.  Epilogue
 * modes as cv3_tc_gemm (0 +bias, 1 GELU-tanh, 2 gated residual, 3 residual). */
int cv3_tc_gemm_q8(const float* a, int64_t lda, const void* w16, const float* scales_t, float* c, int64_t ldc,
                   int64_t m, int64_t n, int64_t k, int mode, const float* bias, const float* gate,
                   int64_t rows_per_group, int64_t gate_stride, void* stream);

/* Activation planes (cv3_tc_gemm_q8_planes' A operand and mode-4 output): an fp32
 * matrix X[m][k] (k % 64 == 0) as planes fp16 [m][2k] -- per row and 64-wide group g,
 * hi = fp16(x * 2^e) at columns 128g..128g+63 and lo = fp16(x * 2^e - hi) at
 * 128g+64..128g+127 -- and exps int8 [k/64][lde] (lde >= m, a multiple of 16), e
 * bringing the group's max |x| into [2^14, 2^15): 22 significant bits per value,
 * the fp32 matrix's bytes.  No counterpart in the reference (an operand format). */

/* cv3_tc_gemm_q8 with A given as activation planes (read by TMA, no conversion in
 * the GEMM).  Modes 0-3 as cv3_tc_gemm_q8 into c; mode 4: GELU-tanh(+bias)
 * written as activation planes (out_planes [m][2n], out_exps [n/64][out_lde]) --
 * the DiT feed-forward's first linear feeding the second (cv3cpu/models/dit.py:
 * 131-142). */
int cv3_tc_gemm_q8_planes(const void* planes, const int8_t* exps, int64_t lde, const void* w16,
                          const float* scales_t, float* c, int64_t ldc, int64_t m, int64_t n, int64_t k, int mode,
                          const float* bias, const float* gate, int64_t rows_per_group, int64_t gate_stride,
                          void* out_planes, int8_t* out_exps, int64_t out_lde, void* stream);

/* fp32 rows x [rows][ldx] -> activation planes (k % 64 == 0). */
int cv3_q8_split_rows(const float* x, int64_t ldx, int64_t rows, int64_t k, void* planes, int8_t* exps,
                      int64_t lde, void* stream);

/* cv3_ln_modulate (dit.py:162-169 AdaLN: LayerNorm without affine, * (1 + scale) +
 * shift) writing activation planes instead of fp32; dim 512 or 1024. */
int cv3_ln_modulate_planes(const float* h, int64_t rows, int64_t dim, float eps, const float* scale,
                           const float* shift, int64_t rows_per_group, int64_t mod_stride, void* planes,
                           int8_t* exps, int64_t lde, void* stream);

/* The operands cv3_tc_gemm_q8 reads, from a q8 matrix (quant.py:90-136 layout,
 * int8 [n][k] with k % 64 == 0, fp16 scales [n][k/64]): w16 fp16 [n][k] (exact)
 * and scales_t fp32 [k/64][n]. */
int cv3_q8_gemm_prepare(const int8_t* q, const uint16_t* scales, int64_t n, int64_t k, void* w16, float* scales_t,
                        void* stream);

/* Error word of cv3_tc_gemm_q8 (see cv3_tc_gemm_status). */
int cv3_tc_gemm_q8_status(int* code);

/* Rearrange conv weights W[C_out][C_in/groups][k] into the tensor-core
 * layout Wt[C_out][ci_pad/32][k][32] (ci_pad = C_in/groups rounded up to 32, zero
 * filled) and, if wt_lo is not NULL, the tf32 remainders.  Done once per
 * weight; weights that are exact tf32 values (fp16-stored) need no remainder. */
int cv3_conv_weight_tc(const float* w, int64_t cout, int64_t cin_g, int64_t k, int64_t ci_pad, float* wt,
                       float* wt_lo, void* stream);

/* cv3_conv1d on the tensor cores (implicit GEMM, tcgen05, 3xTF32 -- 2 products
 * when wt_lo is NULL).  x and y are strided: element (b, c, t) at
 * b*s_b + c*s_c + t*s_t, so channel-major and token-major signals are read and
 * written in place; inputs outside [0, t_in) count as zero padding (t_out sets
 * the right pad).  Epilogue, in order: + bias, activation `act` (-1 none,
 * CV3_ACT_MISH, _ELU or _LEAKY_RELU; parameter act_param), snake with per-output-channel snake_alpha
 * (NULL none; cv3cpu/models/hift.py Snake), + residual (y's strides, may alias
 * y).  Replaces cv3cpu/ops.py:165-219 (conv1d) and the elementwise ops after it. */
int cv3_conv1d_tc(const float* x, int64_t xsb, int64_t xsc, int64_t xst, int64_t batch, int64_t cin, int64_t t_in,
                  const float* wt, const float* wt_lo, int64_t ci_pad, int64_t cout, int64_t k, int64_t stride,
                  int64_t dilation, int64_t groups, int64_t pad_left, const float* bias, int act, float act_param,
                  const float* snake_alpha, const float* residual, float* y, int64_t ysb, int64_t ysc, int64_t yst,
                  int64_t t_out, void* stream);

/* Error word of the tensor-core conv kernel (see cv3_tc_gemm_status). */
int cv3_tc_conv_status(int* code);

/* Programmatic dependent launch of the LM decode step's kernels (q8 decode
 * GEMVs, RoPE + cache append, decode attention, head select, embedding): 1
 * (default) lets each start while the previous kernel on the stream runs --
 * it streams its weights, then waits for the previous kernel's results and
 * only then releases its own successor; 0 launches them normally.  Results
 * are identical; graphs captured afterwards keep the setting. */
int cv3_set_dependent_launch(int enable);

/* Input path of cv3_conv1d_tc: 1 (default) stages each channel block's input
 * window in shared memory by TMA when the strides allow it (16-byte multiples)
 * and the window fits 256 frames, else gathers from global memory; 0 always
 * gathers.  Both give the same results; the switch exists to test both paths. */
int cv3_conv_tc_set_window(int enable);

/* Input path the last cv3_conv1d_tc launch took: 0 gather, 1 channel-major
 * window, 2 token-major window (-1 before the first launch). */
int cv3_conv_tc_last_path(int* path);

/* Persistent greedy decode of the Qwen2 speech LM (cv3cpu/models/qwen2.py:
 * 139-179 per token, llm.py:114 head + greedy pick; replaces the per-token
 * chain of qwen2.py's ops.* calls): `steps` tokens for a batch of <= 8
 * sequences in ONE cooperative launch (one CTA per SM) -- every layer's q8
 * linears (RMSNorm fused in, bias, RoPE + KV append, GQA attention,
 * residuals, SwiGLU), the final norm, the head, log_softmax / first argmax
 * over the speech tokens, bookkeeping (pos, lens, history[b][*step], *step)
 * and the embedding of the chosen token as the next input.  Each CTA streams
 * its fixed share of every weight matrix into shared memory ahead of the
 * dependency chain; phases hand over through completion counters in `sync`
 * (bounded waits; cv3_decode_status reports an expired wait).
 * State on entry is what cv3_head_select + cv3_embedding leave: h holds the
 * embedded current token at position pos[b], lens[b] = pos[b] + 1.
 * Every matrix is q8 ([rows][kp] int8 + fp16 scales [rows][kp/64]) with
 * kp == its K (hidden <= 1216, inter <= 4864, multiples of 64); gate/up rows
 * interleaved (2i gate_i, 2i+1 up_i); qkv rows = q heads, k heads, v heads;
 * the head padded to a multiple of 16 rows (rows >= vocab are not read back).
 * The per-layer table has CV3_DECODE_LAYER_FIELDS device pointers per layer,
 * in this order: */
#define CV3_DECODE_LAYER_FIELDS 13
/*  0 qkv q8, 1 qkv scales, 2 qkv bias (fp32), 3 input RMSNorm weight,
 *  4 o q8, 5 o scales, 6 gate|up q8, 7 gate|up scales, 8 post-attention RMSNorm
 *  weight, 9 down q8, 10 down scales, 11 K cache, 12 V cache
 * (caches [batch][kv_heads][cap][head_dim] fp32). */
typedef struct cv3_decode_params {
  const void* const* layers; /* device array: n_layers * CV3_DECODE_LAYER_FIELDS pointers */
  int32_t n_layers, batch, hidden, heads, kv_heads, head_dim, inter;
  float eps, scale;       /* RMSNorm eps; attention scale (1/sqrt(head_dim), fp32) */
  int64_t cap;            /* KV cache capacity (positions) */
  const float* cos_table; /* [cap][head_dim] */
  const float* sin_table;
  const float* final_norm;
  const int8_t* head_q;   /* [ceil16(vocab)][hidden] q8 */
  const uint16_t* head_s;
  int32_t vocab, select;  /* head rows; tokens eligible for the greedy pick */
  const void* emb;        /* next-token embedding table: fp32 [rows][hidden] or q8 */
  const uint16_t* emb_scales; /* NULL for fp32 */
  int32_t emb_rows;
  float* h;               /* [batch][hidden] residual stream / input */
  float* h1;              /* [batch][hidden] scratch: residual after attention */
  float* qkv;             /* [batch][(heads + 2 kv_heads) * head_dim] scratch */
  float* attn_part;       /* [batch][heads][ceil(cap / 64)][head_dim + 2] scratch (cap <= 1536) */
  float* attn;            /* [batch][heads * head_dim] scratch */
  float* part;            /* scratch: max([hidden/16][ceil(inter/1216)][16][8], [8][ceil(vocab/16)][4]) floats */
  int64_t part_floats;
  float* act;             /* [batch][inter] scratch */
  float* logits;          /* [batch][vocab] */
  float* logp;            /* [batch][vocab] log-probs of the last step, or NULL */
  int32_t* pos;
  int32_t* lens;
  int64_t* next_ids;
  int64_t* history;       /* [batch][hist_stride] */
  int64_t hist_stride;
  int32_t* step;          /* history column of the next token */
  uint32_t* sync;         /* cv3_decode_sync_words() words, zeroed once before the first call */
  int64_t sync_words;
  int32_t steps;
  int32_t trace_step;     /* with trace: the step (of this launch) to record */
  uint64_t* trace;        /* NULL, or [SMs][5 n_layers + 2][6] per-phase timestamps (see decode_stream.cu) */
} cv3_decode_params;

int cv3_decode_steps(const cv3_decode_params* params, void* stream);

/* Words of the `sync` buffer cv3_decode_steps needs for this geometry. */
int64_t cv3_decode_sync_words(int64_t n_layers, int64_t hidden);

/* Error word of the persistent decode kernel (see cv3_tc_gemm_status): 1 a
 * completion wait expired, 2 a position past the cache, 3 a step past the
 * history, 4/5 a weight-ring wait expired, 6 a key/value prefetch wait expired,
 * 7 a token outside the embedding table. */
int cv3_decode_status(int* code);


/* Error word of the tensor-core kernels (0 = none; else the code of the
 * first bounded wait that expired), read and cleared.  Synchronises. */
int cv3_tc_gemm_status(int* code);

/* Same for the tensor-core attention kernel (cv3_attention, head dim 64). */
int cv3_tc_attention_status(int* code);

#ifdef __cplusplus
}
#endif

#endif /* CV3CUDA_H */

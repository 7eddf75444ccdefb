/*
 * qlin -- C ABI of the B200 (sm_100a) quantised-linear hot path.
 *
 * Every entry point replaces one Python/Triton entry point of the reference
 * engine's kernel layer (paths relative to the reference project root; the
 * citation is given per function).  The Python mirror in
 * qwen_3.5_comfy_prompt_enhancer_b200/kernels/{gemm,w4,norm}.py keeps the
 * reference's names, argument order and in-place/return conventions and calls
 * these functions; callers in other languages bind them directly.
 *
 * Conventions shared by every entry point
 *  - All pointers are device pointers on the current CUDA device.  bf16 data is
 *    passed as `void*` (16-bit IEEE bfloat16, row-major).
 *  - Shapes follow the reference: activations a_q int8 [M, K] contiguous with
 *    one fp32 scale per 64 K elements, a_s [M, K/64] contiguous; W8 weights
 *    int8 [K, N] (N contiguous) with fp32 per-column scales [N]; W4 weights
 *    packed uint8 [K/2, N] (byte j of a column: K = 2j in the low nibble,
 *    K = 2j+1 in the high nibble), bf16 group scales [K/WG, N] and optional
 *    uint8 zeros [K/WG, N] (value = nibble - zero; no zeros means zero = 8).
 *  - Outputs are preallocated by the caller and written in place; `ldo`/`ldr`
 *    are row strides in elements.  `residual` may alias `out`.
 *  - Work is enqueued on `stream` (a cudaStream_t; NULL = legacy default
 *    stream) and returns immediately.  Kernels are launched with programmatic
 *    dependent launch: they begin streaming WEIGHTS before the preceding
 *    kernel on the stream has finished, so weights must not be written by the
 *    kernel launched immediately before on the same stream (they are read-only
 *    model parameters in the engine).  Activations, residuals and outputs are
 *    ordered normally.
 *  - Return value: QLIN_OK or a qlin_status code; qlin_last_error() gives a
 *    thread-local message for the most recent failure.
 *  - Device faults.  Every device-side wait (TMA stages, tensor-core commits,
 *    split-K partial sums, peer arrivals) is bounded in time (2 s, see
 *    qlin_set_wait_limit_ns).  A wait that gives up records a bit in the
 *    device fault word and the kernel returns instead of hanging; its outputs
 *    are then invalid.  Launches are asynchronous, so the launching call has
 *    already returned QLIN_OK: the fault is reported like CUDA's sticky
 *    errors instead, by QLIN_ERR_DEVICE_FAULT from every later entry point on
 *    that device (checked on the host through a mapped pinned word, without
 *    synchronising), until qlin_device_fault(1) clears it.
 *  - Requirements beyond the reference's (checked, reported as
 *    QLIN_ERR_SHAPE / QLIN_ERR_ALIGNMENT): K % 64 == 0 (the reference
 *    silently assumes it, kernels/common.py:5-7), N % 16 == 0, 16-byte
 *    aligned base pointers for a_q and every weight / scale / zero tensor.
 */
#ifndef QLIN_H_
#define QLIN_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  QLIN_OK = 0,
  QLIN_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, bad flag */
  QLIN_ERR_SHAPE = 2,            /* shape not supported by the reference contract */
  QLIN_ERR_ALIGNMENT = 3,        /* pointer or stride alignment */
  QLIN_ERR_UNSUPPORTED = 4,      /* valid request this build cannot run */
  QLIN_ERR_CUDA = 5,             /* CUDA runtime / launch error */
  QLIN_ERR_DEVICE_FAULT = 6      /* a bounded device-side wait gave up */
} qlin_status;

/* Library version (major*10000 + minor*100 + patch). */
int qlin_version(void);

/* Static string for a status code. */
const char* qlin_status_string(int status);

/* Thread-local detail message of the last failing call on this thread. */
const char* qlin_last_error(void);

/* Reads (and if `clear`, resets) the device fault word of the current device:
 * a bitmask of bounded waits that gave up inside qlin kernels since the last
 * clear.  Synchronous; for diagnostics and tests.  Returns -1 on CUDA error. */
int qlin_device_fault(int clear);

/* Sets the bound of every device-side wait of later launches on the current
 * device, in nanoseconds (default 2e9).  For tests of the fault path: with a
 * short bound, a wait that nothing will complete ends quickly.  Not part of
 * the reference's interface. */
int qlin_set_wait_limit_ns(int64_t ns);

/* kernels/gemm.py:60-92 (gemm_i8, W8 branch) and gemm.py:20-57 (kernel):
 *   out[m,n] = bf16( (sum_kb float(int32 dot of block kb) * a_s[m,kb]) * b_s[n]
 *                    (+ residual[m,n]) )                                     */
int qlin_gemm_i8(const int8_t* a_q, const float* a_s, int64_t M, int64_t K,
                 const int8_t* b, const float* b_s, int64_t N,
                 void* out, int64_t ldo, const void* residual, int64_t ldr,
                 void* stream);

/* kernels/w4.py:139-166 (gemm_w4) and w4.py:64-136 (_w4_acc, kernel):
 *   out[m,n] = bf16( sum_sub float(int32 dot of sub-block) * (a_s * ws)
 *                    (+ residual[m,n]) ),  SUB = min(WG, 64).
 * b_z may be NULL (symmetric, zero = 8).  WG = K / rows(b_s) is passed as
 * `wgrp` and must be 32 or a multiple of 64. */
int qlin_gemm_w4(const int8_t* a_q, const float* a_s, int64_t M, int64_t K,
                 const uint8_t* b, const void* b_s, const uint8_t* b_z, int64_t N, int64_t wgrp,
                 void* out, int64_t ldo, const void* residual, int64_t ldr,
                 void* stream);

/* kernels/gemm.py:290-312 (proj3) and gemm.py:234-287 (kernel): three W8
 * projections sharing A, written to out[:, 0:n1], [n1:n1+n2], [n1+n2:...].
 * A segment with n_i == 0 is skipped (its pointers may be NULL). */
int qlin_proj3(const int8_t* a_q, const float* a_s, int64_t M, int64_t K,
               const int8_t* w1, const float* s1, int64_t n1,
               const int8_t* w2, const float* s2, int64_t n2,
               const int8_t* w3, const float* s3, int64_t n3,
               void* out, int64_t ldo, void* stream);

/* kernels/w4.py:220-251 (proj3_w4) and w4.py:169-217 (kernel).  Per-segment
 * zeros z_i may be NULL (that segment decodes with zero = 8). */
int qlin_proj3_w4(const int8_t* a_q, const float* a_s, int64_t M, int64_t K,
                  const uint8_t* w1, const void* s1, const uint8_t* z1, int64_t n1,
                  const uint8_t* w2, const void* s2, const uint8_t* z2, int64_t n2,
                  const uint8_t* w3, const void* s3, const uint8_t* z3, int64_t n3,
                  int64_t wgrp, void* out, int64_t ldo, void* stream);

/* kernels/gemm.py:140-151 (mlp_gate_up) and gemm.py:95-137 (kernel):
 *   out = bf16( silu(g * sg) * (u * su) ), out row stride ldo. */
int qlin_mlp_gate_up(const int8_t* a_q, const float* a_s, int64_t M, int64_t K,
                     const int8_t* wg, const float* sg, const int8_t* wu, const float* su,
                     int64_t N, void* out, int64_t ldo, void* stream);

/* kernels/gemm.py:214-231 (mlp_gate_up_quant) and gemm.py:154-211 (kernel):
 *   h = bf16_round( silu(g * sg) * (u * su) );  per (m, 64-column group):
 *   s = max(amax|h| / 127, 1e-8), q = round_half_away(h / s) clamped to +-127.
 * out_q int8 [M, N] contiguous, out_s fp32 [M, N/64] contiguous; N % 64 == 0. */
int qlin_mlp_gate_up_quant(const int8_t* a_q, const float* a_s, int64_t M, int64_t K,
                           const int8_t* wg, const float* sg, const int8_t* wu, const float* su,
                           int64_t N, int8_t* out_q, float* out_s, void* stream);

/* kernels/w4.py:300-323 (mlp_gate_up_quant_w4) and w4.py:254-297 (kernel):
 * as above with W4 weights (scales applied per sub-block inside the K loop). */
int qlin_mlp_gate_up_quant_w4(const int8_t* a_q, const float* a_s, int64_t M, int64_t K,
                              const uint8_t* wg, const void* sg, const uint8_t* zg,
                              const uint8_t* wu, const void* su, const uint8_t* zu,
                              int64_t N, int64_t wgrp, int8_t* out_q, float* out_s,
                              void* stream);

/* kernels/norm.py:75-92 (quant_row) and norm.py:15-25 (_quant_groups):
 * bf16 x [M, K] (row stride ldx) -> int8 q [M, K], fp32 s [M, K/64]:
 *   s = max(amax / 127, 1e-8) (IEEE division), q = round_half_away(x / s). */
int qlin_quant_row(const void* x, int64_t ldx, int64_t M, int64_t K,
                   int8_t* q, float* s, void* stream);

/* ---- Activation producers (kernels/norm.py): they write the (a_q, a_s) that
 * the GEMMs above consume.  Integer codes and scales follow norm.py:15-25
 * exactly given the fp32 value being quantised; that value comes from fp32
 * sums whose order is the kernel's own (the reference's is its compiler's).
 * Inputs need 16-byte aligned rows unless stated otherwise. ---- */

/* kernels/norm.py:28-57 (rmsnorm_quant): per row of bf16 x [M, K] (row
 * stride ldx), var = sum(x^2)/K, y = x * rsqrt(var + eps) * (w + 1 if
 * one_plus else w) with w bf16 [K], then per-64 quantisation into int8 q
 * [M, K] and fp32 s [M, K/64] (both contiguous).  K % 64 == 0, K <= 16384. */
int qlin_rmsnorm_quant(const void* x, int64_t ldx, const void* w, int64_t M, int64_t K, float eps,
                       int one_plus, int8_t* q, float* s, void* stream);

/* kernels/norm.py:95-137 (norm_gated_quant): per (token t, head h) of bf16
 * v [T, N] (contiguous, N = heads * HD), gate z [T, >= N] (row stride ldz)
 * and bf16 w [HD]: y = x * rsqrt(mean(x^2) + eps) * w * silu(z), rounded
 * through bf16, then per-64 quantisation within the head into q [T, N],
 * s [T, N/64].  HD in {64, 128, 256}; 4-byte alignment suffices. */
int qlin_norm_gated_quant(const void* v, const void* z, int64_t ldz, const void* w, int64_t T, int64_t N,
                          int64_t HD, float eps, int8_t* q, float* s, void* stream);

/* kernels/norm.py:141-165 (norm_gated): the same y stored as bf16 out [T, N]. */
int qlin_norm_gated(const void* v, const void* z, int64_t ldz, const void* w, int64_t T, int64_t N,
                    int64_t HD, float eps, void* out, void* stream);

/* kernels/norm.py:168-188 (gate_mul_quant): y = a * sigmoid(g_gate) for bf16
 * a [M, N] (contiguous), where the gate of column n is column
 * (n / hd) * 2 hd + hd + n % hd of the bf16 row g (row stride ldg, the q
 * projection with its per-head gate halves), then per-64 quantisation into
 * q [M, N], s [M, N/64]. */
int qlin_gate_mul_quant(const void* a, const void* g, int64_t ldg, int64_t M, int64_t N, int64_t hd,
                        int8_t* q, float* s, void* stream);

/* kernels/norm.py:191-208 (silu_mul_quant): y = silu(g) * u for bf16 g, u
 * [M, N] (contiguous), then per-64 quantisation into q [M, N], s [M, N/64]. */
int qlin_silu_mul_quant(const void* g, const void* u, int64_t M, int64_t N, int8_t* q, float* s,
                        void* stream);

/* kernels/norm.py:211-240 (gate_proj): from int8 activations a_q [M, K] with
 * per-64 scales a_s [M, K/64], x = a_q * a_s; b = wb @ x, av = wa @ x for
 * bf16 wb, wa [NB, K]; beta = sigmoid(b),
 * gate = -exp(a_log) * softplus(av + dt_bias) with bf16 dt_bias, a_log [NB];
 * beta, gate fp32 [M, NB].  a_q needs 8-byte alignment, wb / wa 16-byte. */
int qlin_gate_proj(const int8_t* a_q, const float* a_s, int64_t M, int64_t K, const void* wb, const void* wa,
                   int64_t NB, const void* dt_bias, const void* a_log, float* beta, float* gate, void* stream);

/* ---- Decode-step neighbours (kernels/attention.py, kernels/linear_attn.py):
 * the kernels between the projections of one decode step.  A position may be
 * passed in device memory (pos_dev, int32; NULL: use the scalar) so that a
 * decode step can be captured in a CUDA graph once and replayed at every
 * position.  bf16 data is 16-byte aligned with row strides in elements. ---- */

/* kernels/attention.py:70-133 (qk_norm_rope) and :20-67 (_norm_rope_store).
 * proj bf16 [T, ldp]: per q head hd query dims then hd gate dims, then nkv k
 * heads, then nkv v heads.  q and k: RMSNorm over hd with (1 + qn / kn), then
 * rotate-half RoPE on the first rd dims at angle pos * invf[i] (invf fp32
 * [rd/2]); q scaled by 1/sqrt(hd) into qout [T, nq*hd].  k and v go to cache
 * row `pos` of kvc [rows, 2*nkv*hd] (k heads then v heads): bf16, or
 * (kv_int8) int8 codes with one fp32 scale max(amax/127, 1e-8) per
 * (position, head, side) in kvs [rows, 2*nkv].  Row t of proj is position
 * pos0 + t, or with `batch` candidate t at position pos0 in its own cache
 * slice starting at t * kv_stride (t * kvs_stride for the scales).
 * hd in {128, 256}. */
int qlin_qk_norm_rope(const void* proj, int64_t ldp, const void* qn, const void* kn, const float* invf,
                      int64_t rd, void* qout, void* kvc, float* kvs, int64_t T, int64_t nq, int64_t nkv,
                      int64_t hd, int64_t pos0, const int32_t* pos_dev, float eps, int kv_int8, int batch,
                      int64_t kv_stride, int64_t kvs_stride, void* stream);

/* kernels/attention.py:209-267 (attn_decode): for each candidate b and q head
 * h, softmax(q_h . k_n) over cache positions n = 0..pos (q already scaled)
 * weighted sum of v_n, bf16 out [batch, nq*hd].  KV head of h: h / (nq/nkv).
 * Cache as written by qlin_qk_norm_rope; candidate b's rows start at
 * b * kv_stride.  max_pos (with pos_dev): the largest position a replay will
 * see, which sets how the positions are split over the CTAs. */
int qlin_attn_decode(const void* q, const void* kvc, const float* kvs, void* out, int64_t pos,
                     const int32_t* pos_dev, int64_t max_pos, int64_t batch, int64_t nq, int64_t nkv,
                     int64_t hd, int kv_int8, int64_t kv_stride, int64_t kvs_stride, void* stream);

/* kernels/linear_attn.py:172-207 (delta_decode): one new token per candidate.
 * qkv bf16 [batch, ldq] holds q [nh*dk], k [nh*dk], v [nh*dv]; g, beta fp32
 * [batch, nh]; state fp32 [batch*nh, dk, dv] updated in place:
 *   qn = q rsqrt(|q|^2 + 1e-6) / sqrt(dk), kn = k rsqrt(|k|^2 + 1e-6),
 *   S *= exp(g); delta = (v - kn^T S) beta; S += kn delta^T; out = qn^T S
 * -> bf16 out [batch, nh*dv].  dk = dv = 128. */
int qlin_delta_decode(const void* qkv, int64_t ldq, const float* g, const float* beta, float* state, void* out,
                      int64_t batch, int64_t nh, int64_t dk, int64_t dv, void* stream);

/* kernels/linear_attn.py:10-47 (conv_silu): depthwise causal conv of width
 * ks = 4 with bf16 weights w [C, 4], then SiLU: bf16 x [T, C] (row stride
 * ldx) -> y [T, C].  Sequence mode: the taps before row 0 read the 3 state
 * rows state [3, C].  Batch mode: row t is candidate t, taps 0..2 read its
 * state rows state[3t .. 3t+2], tap 3 its input row.  C % 8 == 0. */
int qlin_conv_silu(const void* x, int64_t ldx, const void* w, int64_t ks, const void* state, void* y, int64_t T,
                   int64_t C, int batch, void* stream);

/* kernels/linear_attn.py:50-83 (conv_state_update): the conv window keeps the
 * last 3 raw input rows.  batch == 1: state [3, C] <- the last 3 of the T new
 * rows (older state rows when T < 3).  batch > 1 (= T): each candidate's rows
 * state[3b .. 3b+2] shift down by one and take x row b as the newest. */
int qlin_conv_state_update(const void* x, int64_t ldx, void* state, int64_t T, int64_t C, int64_t ks,
                           int64_t batch, void* stream);

/* qlin_conv_silu (batch mode) followed by qlin_conv_state_update (batch mode)
 * of one decode step in one launch: y [batch, C] and the shifted windows
 * state [3*batch, C], identical to the two calls.  No reference counterpart
 * (the engine calls the two kernels back to back, engine.py:302-303). */
int qlin_conv_silu_update(const void* x, int64_t ldx, const void* w, int64_t ks, void* state, void* y,
                          int64_t batch, int64_t C, void* stream);

/* ---- Prefill neighbours ---- */

/* kernels/attention.py:136-206 (attn_prefill): causal attention of T query
 * rows q [T, nq*hd] (bf16, already scaled) at positions pos0 .. pos0 + T - 1
 * over cache rows 0 .. pos0 + t of kvc [rows, 2*nkv*hd] (bf16, or int8 with
 * kvs [rows, 2*nkv], dequantised to bf16(code * scale) as the reference
 * does); bf16 products, fp32 accumulation and softmax, P rounded to bf16 for
 * the P V product -> bf16 out [T, nq*hd].  hd in {128, 256}. */
int qlin_attn_prefill(const void* q, const void* kvc, const float* kvs, void* out, int64_t T, int64_t pos0,
                      int64_t nq, int64_t nkv, int64_t hd, int kv_int8, void* stream);

/* kernels/linear_attn.py:86-169 (delta_prefill): chunked (32 tokens) gated
 * delta rule over T tokens of qkv bf16 [T, ldq] (q [nh*dk], k [nh*dk],
 * v [nh*dv]), g / beta fp32 [T, nh], state fp32 [nh, dk, dv] updated in
 * place; per chunk the WY form with the Neumann-product inverse of the
 * reference, in fp32 -> bf16 out [T, nh*dv].  dk = 128, dv % 32 == 0. */
int qlin_delta_prefill(const void* qkv, int64_t ldq, const float* g, const float* beta, float* state, void* out,
                       int64_t T, int64_t nh, int64_t dk, int64_t dv, void* stream);

/* ---- Multi-GPU (column-split layer): NVLink peer memory through CUDA IPC ----
 * Not part of the reference's interface (it has no multi-GPU path); used by
 * the package's tp.py for its all-gathers. */
#define QLIN_IPC_HANDLE_BYTES 64

/* IPC handle (QLIN_IPC_HANDLE_BYTES bytes) of the allocation holding device
 * pointer `ptr`, and the byte offset of `ptr` inside it. */
int qlin_ipc_get_handle(const void* ptr, void* handle, int64_t* offset);

/* Opens a peer's handle in this process; *ptr = mapped base + offset. */
int qlin_ipc_open(const void* handle, int64_t offset, void** ptr);

/* Closes a mapping opened by qlin_ipc_open (same ptr and offset). */
int qlin_ipc_close(void* ptr, int64_t offset);

/* Zero-filled device allocation of its own (one IPC handle per buffer). */
int qlin_dev_alloc(int64_t bytes, void** ptr);
int qlin_dev_free(void* ptr);

/* All-gather of `shard_bytes` (multiple of 16) from `src` into slot `rank` of
 * every rank's buffer bufs[q] (world x shard_bytes bytes each), then waits
 * until every rank's shard has landed in bufs[rank]; if `dst` is not null the
 * gathered world x shard_bytes bytes are then copied there on the same
 * stream.  arrive[q] is rank q's array of `world` uint32 arrival counters
 * (zero-initialised once, never reset); `expected` is this rank's device
 * array of `world` uint32 (zero once).  Every rank must call it with the same
 * shard_bytes.  A wait that does not finish within 2 s sets the device fault
 * word. */
int qlin_peer_allgather(void* const* bufs, void* const* arrive, void* expected, const void* src,
                        int64_t shard_bytes, int world, int rank, void* dst, void* stream);

/* One 2-D block of this rank's data for qlin_peer_allgather_ll: `rows` rows
 * of `row_bytes` bytes, `src_ld` bytes apart.  Rank q's block lands in every
 * rank's destination at byte dst_off + q * row_bytes, rows dst_ld bytes apart
 * -- so a shard of output COLUMNS goes straight into its column range of a
 * row-major [rows, world * row_bytes / element size] matrix.  row_bytes,
 * dst_off and dst_ld must be multiples of 4 (multiples of 8 move twice the
 * data per store); the source, its stride and the destination must be
 * aligned to the same 8 or 4 bytes. */
typedef struct {
  const void* src;
  int64_t src_ld;
  int64_t rows;
  int64_t row_bytes;
  int64_t dst_off;
  int64_t dst_ld;
} qlin_gather_part;

/* Words of the per-rank state array of qlin_peer_allgather_ll. */
#define QLIN_PEER_STATE_WORDS 16

/* Bytes of the exchange buffer every rank needs for qlin_peer_allgather_ll
 * with these parts at `world` ranks (twice the data of all ranks, twice over
 * for the two alternating halves).  No GPU needed. */
int qlin_peer_ll_bytes(const qlin_gather_part* parts, int nparts, int world, int64_t* bytes);

/* All-gather of one to four 2-D parts (qlin_gather_part) into `dst`, this
 * rank's destination, on every rank.  ll[q] is rank q's exchange buffer
 * (this rank's own at [rank], the others opened through CUDA IPC), at least
 * ll_bytes >= qlin_peer_ll_bytes(...) bytes, 16-byte aligned and zeroed once;
 * `state` is this rank's device array of QLIN_PEER_STATE_WORDS uint32, zeroed
 * once.  Every 8-byte word a rank stores into a peer's exchange buffer
 * carries the call's sequence number beside 4 data bytes, so the receiving
 * kernel knows a word has landed by reading it: no fence, counter or second
 * round trip stands between the stores and the data's use, which is what
 * makes this the low-latency form for the few-KB gathers of a decode step.
 * The kernel copies this rank's blocks into its own slots of dst, stores them
 * into every peer's exchange buffer, then waits for every peer's words and
 * writes them into the peers' slots of dst.  Every rank must call it with the
 * same sizes, the same number of times, in the same order for the same
 * buffers.  A wait that does not finish within the wait limit records a
 * device fault.  Not part of the reference's interface (it has no multi-GPU
 * path); the column-split layer (tp.py) gathers its h codes + scales and its
 * output with it. */
int qlin_peer_allgather_ll(void* const* ll, int64_t ll_bytes, void* state, const qlin_gather_part* parts,
                           int nparts, int world, int rank, void* dst, void* stream);

/* All-gather of one or two 2-D parts (qlin_gather_part) straight into every
 * rank's gather buffer bufs[q] (each holding dst_off + (rows - 1) * dst_ld +
 * world * row_bytes bytes for every part), then a wait until every rank's
 * parts have landed in bufs[rank]: the arrival-counter protocol of
 * qlin_peer_allgather (plain stores, one system-scope fence and release per
 * CTA, counters in every rank's memory).  It moves each byte once where the
 * flagged words of qlin_peer_allgather_ll move it twice, so large gathers
 * (hundreds of KB per rank and up) take it.  arrive[q]: rank q's `world`
 * uint32 arrival counters (zero once); `expected`: this rank's `world` uint32
 * (zero once).  Sizes, strides and addresses multiples of 4 (16 for full-width
 * stores).  Every rank must call it with the same sizes.  A wait that does not
 * finish within the wait limit records a device fault.  No reference
 * counterpart. */
int qlin_peer_allgather_fenced(void* const* bufs, void* const* arrive, void* expected, const qlin_gather_part* parts,
                               int nparts, int world, int rank, void* stream);

/* The two halves of qlin_peer_allgather_ll, for a gather whose sending or
 * receiving side sits inside another kernel (the column-split layer's down
 * projection, qlin_tp_gemm_w4_ll).  qlin_peer_ll_send stores this rank's
 * parts as flagged words of call state[0] + 1 into every rank's exchange
 * buffer, this rank's own included, and advances nothing.  qlin_peer_ll_recv
 * waits for every rank's words of call state[0] + 1 (own included) and writes
 * them into their slots of dst; its last CTA then stores that call number in
 * state[0] and, if state2 is not null, adds one to state2[0] (the call count
 * of a buffer whose readers finished before this launch).  Same layouts,
 * sizes and rules as qlin_peer_allgather_ll.  No reference counterpart. */
int qlin_peer_ll_send(void* const* ll, int64_t ll_bytes, void* state, const qlin_gather_part* parts, int nparts,
                      int world, int rank, void* stream);
int qlin_peer_ll_recv(void* const* ll, int64_t ll_bytes, void* state, const qlin_gather_part* parts, int nparts,
                      int world, int rank, void* dst, void* state2, void* stream);

/* The column-split layer's W4 down projection (kernels/w4.py:139-166
 * gemm_w4, without residual) for 1-4 rows with both all-gathers around it
 * inside the kernel: the activation rows h [M, K] and their scales come from
 * the ranks' flagged words in this rank's exchange buffer of h (h_ll[rank],
 * sent by qlin_peer_ll_send with h_parts = [codes rows M x K/world bytes,
 * scales rows M x K/world/64 floats], call h_state[0] + 1), and every row of
 * this rank's output [M, N] goes to out (row stride ldo) and, as flagged words
 * of call o_state[0] + 1, to every rank's exchange buffer of the output
 * (o_ll, o_parts = [rows M x 2N bytes]) for qlin_peer_ll_recv.  hq / hs, if
 * not null, receive a copy of the gathered h and scales.  K / world must be a
 * multiple of 128.  Returns QLIN_ERR_UNSUPPORTED if the decode-row kernel has
 * no plan for the shape (qlin_plan_dp); the caller then uses the separate
 * gathers.  No reference counterpart (the reference has no multi-GPU path). */
int qlin_tp_gemm_w4_ll(int64_t M, int64_t K, const uint8_t* b, const void* b_s, const uint8_t* b_z, int64_t N,
                       int64_t wgrp, void* out, int64_t ldo, void* const* h_ll, int64_t h_ll_bytes, const void* h_state,
                       const qlin_gather_part* h_parts, int h_nparts, void* const* o_ll, int64_t o_ll_bytes,
                       const void* o_state, const qlin_gather_part* o_parts, int o_nparts, int world, int rank,
                       void* hq, void* hs, void* stream);

/* Diagnostic: the decode-row (dp4a) kernel's plan for wbits 8 or 4, one
 * output stream (gate_up 0) or the fused gate/up (1), M rows, K, `tiles`
 * 128-column tiles, W4 group size and `sms` SMs (0: the current device).
 * out[0..3] = cluster split, K parts across clusters, weight-ring slots per
 * warp (0: resident), 64-K groups per CTA; all zero if the shape goes to the
 * tensor-core kernels.  No GPU needed when sms > 0. */
int qlin_plan_dp(int wbits, int gate_up, int64_t M, int64_t K, int64_t tiles, int64_t wgrp, int sms, int64_t* out);

/* All-gather that allocates nothing, for one rank.  It has no counterpart in
 * the reference.  Meant for a process that runs the column-split layer on a
 * single GPU (world = 1) and may not call cudaMalloc itself -- for instance a
 * plugin whose host application owns all device memory through its own pool,
 * so any allocation of ours would escape that pool's accounting and limits.
 * It runs the same kernel as qlin_peer_allgather with world = 1, but its
 * gather buffer and counters are static device arrays of this library on the
 * current GPU; the caller passes only its shard and the output.
 *   src: shard_bytes bytes (multiple of 16, 16-byte aligned);
 *   dst: shard_bytes bytes, the gathered result, written on `stream`.
 * Limit: shard_bytes <= QLIN_STATIC_GATHER_MAX_BYTES; larger requests fail
 * with QLIN_ERR_SHAPE before anything is launched.  The first call on a
 * device looks up the static arrays' device addresses, so make it before any
 * stream capture.  Every call on a device shares the same arrays: calls on
 * one stream are ordered, calls that overlap on the GPU (other streams) race.
 * The counters start at zero when the library loads and only grow, so nothing
 * is cleared per call.  Its wait is bounded like every other: if it gives up,
 * the call has still returned QLIN_OK and dst holds stale bytes; the fault
 * word says so (qlin_device_fault, and QLIN_ERR_DEVICE_FAULT from later entry
 * points once any other entry point has run on the device and set up the
 * host-visible mirror -- this one allocates nothing, not even that).  (It serves one GPU: a two-GPU form, whose kernels
 * wrote the other GPU's static arrays through peer access, stopped with an
 * illegal memory access on B200, so multi-GPU gathers use
 * qlin_peer_allgather and its caller-allocated buffers.) */
#define QLIN_STATIC_GATHER_MAX_BYTES (4 << 20)
int qlin_peer_allgather_static(const void* src, int64_t shard_bytes, void* dst, void* stream);

/* Diagnostic (no GPU needed, nothing launched): the launch plan of the
 * small-M weight-streaming kernel for wbits 8 or 4, `gate_up` 0 (one output
 * stream: gemm / proj3) or 1 (fused gate/up), M rows, K, `tiles` 128-column
 * output tiles (sum over proj3 segments), W4 group size and `sms` SMs.
 * out[0..9] = K split (cluster size), 64-K groups per CTA, groups per batch,
 * weight-ring slots, unpacked-ring slots, accumulator buffers, dynamic
 * shared memory bytes, activation rows per row block, 1 if the split-K
 * partial sums reuse rank 0's operand region, plan level (2: one batch,
 * 0: streamed).  With sms > 0 it needs no GPU: clusters are counted by
 * shared-memory slots, whereas a launch also checks the device's
 * resident-cluster capacity (qlin_max_active_clusters) and may then choose
 * another split.  sms = 0 gives exactly the plan a launch on the current
 * device gets. */
int qlin_plan_small_m(int wbits, int gate_up, int64_t M, int64_t K, int64_t tiles, int64_t wgrp,
                      int sms, int64_t* out);

/* Diagnostic: clusters of `split` CTAs with `smem` bytes of dynamic shared
 * memory that the current device keeps resident at once, for the small-M
 * kernel instance serving (wbits, gate_up, M)
 * (cudaOccupancyMaxActiveClusters).  Needs a CUDA device. */
int qlin_max_active_clusters(int wbits, int gate_up, int64_t M, int split, int64_t smem, int64_t* out);

#ifdef __cplusplus
}
#endif

#endif /* QLIN_H_ */

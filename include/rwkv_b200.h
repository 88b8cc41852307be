/*
 * rwkv_b200.h -- C ABI of the B200 (sm_100a) WKV-7 and LoRA-MoE kernels.
 *
 * Every entry point takes plain device pointers, sizes and an opaque CUDA
 * stream (cudaStream_t passed as void*; NULL = legacy default stream).  Work is
 * enqueued on that stream; no entry point synchronises the host.  The caller
 * allocates every input, output and workspace buffer.  Return value: 0 on
 * success, otherwise a rwkv_status code (a launch failure is reported as
 * RWKV_ERR_CUDA; rwkv_last_error() gives the CUDA error string).
 *
 * Conventions shared by the WKV-7 entry points (reference:
 * rwkv_mlx/kernels/wkv7_metal.py:250-319):
 *   - per-token tensors r, w, k, v, a, b, y, dy and the six gradients are
 *     (B, T, H, N) row-major, i.e. (B, T, C) with C = H*N, in `dtype`;
 *   - w is the log-log decay: the per-step decay is exp(-exp(w))
 *     (wkv7_metal.py:57) unless stated otherwise; w has its own dtype code
 *     `w_dtype`, either equal to `dtype` or RWKV_F32 (the reference model
 *     promotes w to fp32 through its fp32 bias w0, model.py:200, and the Metal
 *     kernel reads each input in its own dtype);
 *   - states are float32 (B, H, N, N), row i = value index, column j = key
 *     index; one step is  S <- S diag(decay) + (S a) b^T + v k^T,  y = S r;
 *   - N (head size) must be 64 (the reference asserts the same,
 *     rwkv_mlx/model.py:115).
 */
#ifndef RWKV_B200_H
#define RWKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    RWKV_OK = 0,
    RWKV_ERR_SHAPE = 1,     /* a size is <= 0, inconsistent or too large */
    RWKV_ERR_DTYPE = 2,     /* unsupported dtype code */
    RWKV_ERR_HEAD_SIZE = 3, /* N != 64 */
    RWKV_ERR_CUDA = 4,      /* a CUDA call or launch failed */
    RWKV_ERR_ALIGN = 5,     /* a pointer is not aligned as required */
    RWKV_ERR_ARG = 6,       /* a required pointer is NULL or an option is invalid */
    RWKV_ERR_WORKSPACE = 7  /* workspace smaller than the *_workspace_size query */
} rwkv_status;

typedef enum { RWKV_F32 = 0, RWKV_F16 = 1, RWKV_BF16 = 2 } rwkv_dtype;

/* Human-readable text of the last CUDA error seen by this library (per thread). */
const char* rwkv_last_error(void);
/* ABI version of this header (bumped on any signature change). */
int rwkv_abi_version(void);
/* Error word set by a kernel that gave up a bounded wait (0 = none).  Reads the
 * device word synchronously; `clear` resets it.  Negative on a CUDA error.
 * A CTA of the tcgen05 WKV-7 forward that gives up also fills its outputs (y, sa,
 * sT, ckpt) with NaN, so an abort never leaves plausible-looking values behind.
 * No counterpart in the reference (its Metal kernels have no waits). */
int rwkv_device_error(int clear);
/* Test hooks, no counterpart in the reference: make every bounded wait of the
 * tcgen05 WKV-7 forward give up at once (on != 0), exercising its abort path
 * without any real stall; set the device error words of the tcgen05 WKV-7 forward
 * and of the chunked backward directly (a chunked backward that finds its word set
 * writes NaN gradients: its first pass gave up, or an earlier error is unread).  */
int rwkv_debug_force_wait_timeout(int on);
int rwkv_debug_set_device_error(int value);
/* Select the WKV-7 forward kernel: 0 automatic (with all per-token inputs 16-byte
 * aligned: the tcgen05 kernel for fp16/bf16 activations, the mma.sync kernel for
 * fp32; otherwise the step-sequential kernel), 1 step-sequential, 2 chunked on
 * mma.sync, 3 chunked on tcgen05 (fp16/bf16 only).  Process-wide; meant for testing
 * one implementation against another. */
int rwkv_set_wkv_impl(int impl);

/* ------------------------------------------------------------------------ */
/* WKV-7 forward.
 * Replaces wkv7_metal_forward (rwkv_mlx/kernels/wkv7_metal.py:250-279) and the
 * forward kernel body (:28-91).
 *   s0    optional initial state (B,H,N,N) fp32; NULL = zeros (the reference
 *         always starts from zero).
 *   y     output (B,T,H,N) in dtype.
 *   sT    optional final state (B,H,N,N) fp32.
 *   ckpt  optional state snapshots, (B,H,T/ckpt_len,N,N) fp32: snapshot c is
 *         the state after step (c+1)*ckpt_len-1, as the reference writes `s`
 *         every 16 steps (:80-89).  Needed by rwkv_wkv7_backward.
 *   sa    optional (B,T,H,N) fp32: sa_t = S_{t-1} a_t per step (the reference's
 *         `sa_out`, :63-68).
 *   ckpt_len  multiple of 16, >= 16 (ignored when ckpt == NULL).          */
int rwkv_wkv7_forward(const void* r, const void* w, const void* k, const void* v,
                      const void* a, const void* b, const float* s0, void* y,
                      float* sT, float* ckpt, float* sa, int B, int T, int H, int N,
                      int dtype, int w_dtype, int ckpt_len, void* stream);

/* WKV-7 forward with a caller-provided workspace (same contract and reference code
 * as rwkv_wkv7_forward, wkv7_metal.py:250-279 and :28-91).  When B*H leaves most
 * SMs idle, the tcgen05 kernel cuts each sequence into segments of whole 16-step
 * chunks: a transition pass computes every segment's affine state map
 * S_end = S_start M + C (a 128-row state [C; M]), a scan composes them into each
 * segment's initial state, and the forward runs all segments in parallel.  The
 * workspace holds those maps and states: rwkv_wkv7_forward_workspace_size bytes
 * (0 when no segmenting happens for these sizes; workspace may then be NULL).  */
size_t rwkv_wkv7_forward_workspace_size(int B, int T, int H, int N, int dtype);
int rwkv_wkv7_forward_ws(const void* r, const void* w, const void* k, const void* v,
                         const void* a, const void* b, const float* s0, void* y,
                         float* sT, float* ckpt, float* sa, int B, int T, int H, int N,
                         int dtype, int w_dtype, int ckpt_len, void* workspace,
                         size_t workspace_bytes, void* stream);
/* Segments per sequence of rwkv_wkv7_forward_ws and of the chunked backward's
 * adjoint chain (rwkv_wkv7_backward_ws): 0 automatic (default), n >= 1 fixed
 * (capped at the chunk count; the backward keeps segments of at least 3 chunks).
 * Process-wide; meant for testing.  No counterpart in the reference. */
int rwkv_set_wkv_segments(int nseg);

/* WKV-7 backward, exact (no division by the decay).
 * Replaces wkv7_metal_backward (wkv7_metal.py:282-319) and the backward kernel
 * body (:102-214).  The reference reconstructs earlier states by dividing by the
 * decay (:174-178); this entry point recomputes them from `ckpt` instead.
 *   ckpt  snapshots from rwkv_wkv7_forward with the same ckpt_len and s0.
 *   dsT   optional gradient w.r.t. the final state; ds0 optional output.
 *   dr..db outputs (B,T,H,N) in dtype; dw is w.r.t. the log-log w input.   */
int rwkv_wkv7_backward(const void* r, const void* w, const void* k, const void* v,
                       const void* a, const void* b, const void* dy, const float* s0,
                       const float* dsT, const float* ckpt, void* dr, void* dw, void* dk,
                       void* dv, void* da, void* db, float* ds0, int B, int T, int H,
                       int N, int dtype, int w_dtype, int ckpt_len, void* stream);

/* WKV-7 backward, chunked (same contract as rwkv_wkv7_backward, replacing the same
 * reference code, wkv7_metal.py:282-319 and :102-214), with a caller-provided
 * workspace of rwkv_wkv7_backward_workspace_size(B, T, H, N) bytes (fp32 state
 * gradients at every 16-step chunk boundary).  Two launches: the adjoint of the
 * chunk state chain per (b, h), then every chunk's input gradients in parallel.
 * When B*H chains would leave most SMs idle (B*H <= #SMs / 4), the chain is cut into
 * segments: a transition pass computes each segment's affine map of the state gradient
 * (in the workspace's own per-chunk slots), a scan composes them, and all segments run
 * in parallel; the workspace size is the same.
 * Needs ckpt_len == 16 (a snapshot at every chunk boundary); other ckpt_len values,
 * or rwkv_set_wkv_impl(1), run the step-sequential backward of rwkv_wkv7_backward.
 * Precision: the chunk products run on the tensor cores in TF32.  With fp16 / bf16
 * inputs each product is one TF32 product (as in the chunked forward; gradient error
 * ~6e-4 relative to RMS against float64 for fp16); with fp32 inputs each operand is
 * split into two TF32 terms (three products, fp32-level gradients).  */
size_t rwkv_wkv7_backward_workspace_size(int B, int T, int H, int N);
/* Kernels rwkv_wkv7_backward_ws enqueues on the chunked path for these sizes on the
 * current device (2, 4 when segmented, 8 when the chain runs in parts; 0 for invalid
 * sizes), for callers that count launches.  No counterpart in the reference. */
int rwkv_wkv7_backward_launch_count(int B, int T, int H, int N);
int rwkv_wkv7_backward_ws(const void* r, const void* w, const void* k, const void* v,
                          const void* a, const void* b, const void* dy, const float* s0,
                          const float* dsT, const float* ckpt, void* dr, void* dw, void* dk,
                          void* dv, void* da, void* db, float* ds0, int B, int T, int H,
                          int N, int dtype, int w_dtype, int ckpt_len, void* workspace,
                          size_t workspace_bytes, void* stream);

/* One RNN-mode step for Bs independent sequences, state updated in place.
 * Replaces the state update of _time_mixing_rnn (rwkv_mlx/model.py:475-483),
 * batched over sequences (the reference runs one sequence per call).
 *   S      (Bs,H,N,N) fp32, read and written.
 *   r..b   (Bs,H,N) in dtype; y (Bs,H,N) in dtype.
 *   w_mode 0: w is log-log (decay = exp(-exp(w)), as in GPT mode);
 *          1: w is the decay itself (model.py:477 computes it directly). */
int rwkv_wkv7_step(float* S, const void* r, const void* w, const void* k, const void* v,
                   const void* a, const void* b, void* y, int Bs, int H, int N, int dtype,
                   int w_dtype, int w_mode, void* stream);

/* ------------------------------------------------------------------------ */
/* LoRA-MoE router.  Replaces Router.__call__ (rwkv_mlx/moe.py:51-86).
 *   x       (ntok, C) in dtype.      gate_w (E, C) fp32 (nn.Linear weight).
 *   bias    optional (E,) fp32 added to the logits (NULL = reference router).
 *   logits  optional output (ntok, E) fp32.
 *   inds    output (ntok, topk) int32, slots in descending logit order, ties
 *           to the lower expert id (argpartition leaves both unspecified,
 *           moe.py:66-68).
 *   scores  output (ntok, topk) in dtype: softmax over the selected logits.
 *   stats   output fp32[2 + E]: [aux, z, f_0..f_{E-1}] with
 *           aux = E * sum_e f_e p_e, z = mean_t (log sum_e exp l_te)^2
 *           (moe.py:61-62, :76-84).
 *   counts  optional output int32[E]: tokens-slots routed to each expert.
 *   workspace  >= rwkv_moe_router_workspace_size(ntok, E) bytes.
 * Constraints: E <= 32, topk <= E, C % 8 == 0, x 16-byte aligned.          */
size_t rwkv_moe_router_workspace_size(int ntok, int E);
int rwkv_moe_router(const void* x, const float* gate_w, const float* bias, float* logits,
                    int32_t* inds, void* scores, float* stats, int32_t* counts,
                    void* workspace, size_t workspace_bytes, int ntok, int C, int E,
                    int topk, int dtype, void* stream);

/* Same as rwkv_moe_router, but allocates nothing and takes no workspace.
 * No counterpart in the reference: it exists for callers that cannot allocate
 * device memory -- an FFI binding that holds only the buffers a framework handed
 * it, or a serving loop that reserves all device memory at start-up and must not
 * allocate later (cudaMalloc can synchronise the device and fails once memory is
 * reserved).  Its scratch is a file-scope device array of
 * rwkv_moe_router_noalloc_scratch_bytes() bytes (~75 KB), held by every GPU that
 * loads this library until the process exits.  Limit: E <= 32 (any ntok).
 * The first call in a CUDA context looks up that array's device address with
 * the device current (again after a cudaDeviceReset, which makes a new
 * context); make that first call before any stream capture.  All calls
 * on a device share the array (it keeps the last call's contents; nothing in it
 * needs to start at zero), so calls that overlap on the same GPU, e.g. on two
 * streams, race: serialize them. */
size_t rwkv_moe_router_noalloc_scratch_bytes(void);
int rwkv_moe_router_noalloc(const void* x, const float* gate_w, const float* bias,
                            float* logits, int32_t* inds, void* scores, float* stats,
                            int32_t* counts, int ntok, int C, int E, int topk, int dtype,
                            void* stream);

/* Stable counting sort of the (token, slot) routing entries by expert.
 * The reference has no counterpart (it loops densely over all experts,
 * moe.py:139-145); this builds the dispatch order its output is invariant to.
 *   inds     (ntok, topk) int32 expert ids in [0, E).
 *   perm     output int32[ntok*topk]: perm[p] = entry (tok*topk+slot) placed at
 *            sorted position p; entries of one expert keep ascending entry order.
 *   inv      output int32[ntok*topk]: inv[entry] = p.
 *   offsets  output int32[E+1]: expert e owns positions [offsets[e], offsets[e+1]).
 *   workspace >= rwkv_moe_permute_workspace_size(ntok*topk, E) bytes.      */
size_t rwkv_moe_permute_workspace_size(int n_entries, int E);
int rwkv_moe_permute(const int32_t* inds, int32_t* perm, int32_t* inv, int32_t* offsets,
                     void* workspace, size_t workspace_bytes, int ntok, int topk, int E,
                     void* stream);

/* Grouped down-projection of the routed entries: for sorted position p with
 * entry = perm[p], token = entry / topk, expert e (offsets):
 *   h[p, :] = x[token, :] @ A[e]         (moe.py:142, first product)
 *   x (ntok, C) dtype; A (E, C, R) dtype; h (ntok*topk, R) fp32.          */
int rwkv_moe_lora_down(const void* x, const void* A, const int32_t* perm,
                       const int32_t* offsets, float* h, int ntok, int C, int R, int E,
                       int topk, int dtype, void* stream);

/* Combine: out[t] = base[t] + sum_slot scores[t,slot] * (h[inv[t*topk+slot]] @ B[e])
 * with e = inds[t,slot] (moe.py:142-147).  base may equal out (in place) or be
 * NULL (treated as zeros).  B (E, R, C) dtype; out (ntok, C) dtype.        */
int rwkv_moe_lora_combine(const void* base, const float* h, const void* B,
                          const int32_t* inds, const void* scores, const int32_t* inv,
                          void* out, int ntok, int C, int R, int E, int topk, int dtype,
                          void* stream);

/* Fused adapter apply (replaces the two products of moe.py:142 and the weighted
 * sum of moe.py:143-147 in one pass over the tokens):
 *   out[t] = base[t] + sum_s scores[t,s] * ((x[t] @ A[e]) @ B[e]),  e = inds[t,s]
 * Dense over the E*R adapter columns on the tensor cores with the unselected
 * experts masked to 0, which is the reference's own dense formulation.  fp16 / bf16
 * only; needs C % 64 == 0, R % 8 == 0, E*R in {32, 64, 128}, topk <= min(E, 8)
 * (rwkv_moe_lora_apply_supported says whether a shape qualifies).  base and scores
 * may be NULL (zeros / all 1); base may equal out.  x (ntok, C), A (E, C, R),
 * B (E, R, C), out (ntok, C) in dtype; inds (ntok, topk) int32.           */
int rwkv_moe_lora_apply_supported(int C, int R, int E, int topk, int dtype);
int rwkv_moe_lora_apply(const void* x, const void* base, const void* A, const void* B,
                        const int32_t* inds, const void* scores, void* out, int ntok, int C,
                        int R, int E, int topk, int dtype, void* stream);
/* Select the kernel of rwkv_moe_lora_apply: 0 automatic (2, or 1 when the driver cannot
 * build TMA tensor maps), 1 mma.sync (64-token tiles, two passes per tile), 2 tcgen05
 * (persistent, warp-specialised, 128-token tiles, operands moved by TMA into the tensor
 * cores' shared-memory layouts, accumulators in tensor memory).  Process-wide; meant for
 * testing one against the other. */
int rwkv_moe_set_apply_impl(int impl);

/* LoRA-MoE ChannelMix delta with the router folded in (fp16): one pass over x
 * forms the router logits (moe.py:56, x @ W^T with W split into two fp16 terms
 * whose products are exact in fp32, + bias), the top-k routing and scores
 * (moe.py:66-70, ties to the lower expert id, scores in fp16), the aux / z
 * statistics (moe.py:61-84, via the router's fixed-order finalize) and
 *   out = base + sum_s scores[:, s] * (x @ A[e_s]) @ B[e_s]   (moe.py:142-147).
 * Replaces Router.__call__ + the expert loop of LoRAMoE_CMix.__call__
 * (moe.py:51-86, :129-147).  Outputs inds (ntok, topk) int32, scores (ntok,
 * topk) fp16, stats fp32[2 + E] and counts int32[E] as rwkv_moe_router; out may
 * equal base.  Needs rwkv_moe_lora_apply_routed_supported (fp16, E <= 16,
 * E * R in {32, 64, 128}, C % 64 == 0) and a 256-byte aligned workspace of
 * rwkv_moe_lora_apply_routed_workspace_size(ntok, C, E) bytes.  Routing agrees
 * with rwkv_moe_router up to near-ties (a different fp32 summation order).  */
int rwkv_moe_lora_apply_routed_supported(int C, int R, int E, int topk, int dtype);
size_t rwkv_moe_lora_apply_routed_workspace_size(int ntok, int C, int E);
int rwkv_moe_lora_apply_routed(const void* x, const void* base, const void* A, const void* B,
                               const float* gate_w, const float* bias, int32_t* inds, void* scores,
                               float* stats, int32_t* counts, void* workspace,
                               size_t workspace_bytes, void* out, int ntok, int C, int R, int E,
                               int topk, int dtype, void* stream);

/* Expert-parallel dispatch / combine helpers (no counterpart in the reference,
 * which runs on one device; they move the routed rows of moe.py:139-145 between
 * GPUs and back).
 * gather_rows:  rows[p] = x[perm[p] / topk]          (C * sizeof(dtype) % 16 == 0)
 * lora_up:      y[dst] = h[p] @ B[e(p)], e(p) from offsets, dst = out_index[p] (or p
 *               when out_index is NULL); h (n, R) fp32, B (E, R, C), y (n, C) dtype.
 * combine_rows: out[t] = base[t] + sum_s scores[t,s] * rows[inv[t*topk + s]]
 *               (base may be NULL or equal to out).                            */
int rwkv_moe_gather_rows(const void* x, const int32_t* perm, void* rows, int n, int C, int topk,
                         int dtype, void* stream);
int rwkv_moe_lora_up(const float* h, const void* B, const int32_t* offsets,
                     const int32_t* out_index, void* y, int n, int C, int R, int E, int dtype,
                     void* stream);
int rwkv_moe_combine_rows(const void* base, const void* rows, const void* scores,
                          const int32_t* inv, void* out, int ntok, int C, int topk, int dtype,
                          void* stream);

/* Full-expert dispatch (MoE_CMix.__call__, moe.py:231-236, replaces the per-expert
 * token shift and lerp of the dense loop): for sorted position p (rwkv_moe_permute)
 * with tok = perm[p] / topk and e its expert (offsets),
 *   rows[p] = x[tok] + (x_prev - x[tok]) * x_k[e]
 * x_prev = x[tok - 1] inside a sequence of T tokens, prev[tok / T] for the first token
 * of a sequence (prev NULL: zeros, the reference's _time_shift; T = 1 with prev =
 * the stored previous token gives RNN mode).  x (ntok, C), prev (ntok / T, C),
 * x_k (E, C), rows (n = ntok * topk, C), all in dtype, 16-byte aligned,
 * C * sizeof(dtype) % 16 == 0.
 * The expert products then run on rows [offsets[e], offsets[e+1]). */
int rwkv_moe_expert_mix_rows(const void* x, const void* prev, const void* x_k,
                             const int32_t* perm, const int32_t* offsets, void* rows, int n,
                             int T, int C, int topk, int E, int dtype, void* stream);

/* Grouped GEMM on the tcgen05 tensor cores (fp16 / bf16, fp32 accumulation):
 *   out[m, :] = epi(A[m, :] @ W[g]^T) for the rows m in [offs[g], offs[g+1]),
 * the expert products of MoE_CMix.__call__ (moe.py:231-236: key, squared ReLU,
 * value) over the rows that rwkv_moe_expert_mix_rows sorted by expert.  The
 * offsets stay on the device (no host read: the call can be captured in a CUDA
 * graph); offs NULL with G = 1 is a plain GEMM over rows [0, M).
 * A (M, K), W (G, N, K), out (M, ldo) row-major in dtype, 16-byte aligned;
 * K % 8 == 0.  epi 0: the product rounded to dtype; epi 1: relu(.)^2 of the
 * product rounded to dtype (moe.py:234).  Rows outside every group are not written. */
int rwkv_grouped_gemm(const void* a, const void* w, const int32_t* offs, void* out, int M, int N, int K,
                      int G, long long ldo, int epi, int dtype, void* stream);

/* sum_{i<j} ||A_i^T A_j||_F^2 over the expert down-projections
 * (LoRAMoE_CMix.orthogonal_loss, moe.py:149-163).  A (E, C, R) dtype;
 * out: one fp32 scalar.  R <= 64.                                          */
int rwkv_moe_ortho_loss(const void* A, float* out, int E, int C, int R, int dtype,
                        void* stream);

/* ------------------------------------------------------------------------ */
/* Fused element-wise kernels of the block around WKV-7 (the callers defined in
 * rwkv_mlx/model.py:187-263, 312-327).  Activations (rows = B*T, C) in dtype.
 *
 * rwkv_lerp: out[m] = x + (shift(x) - x) * mix[m] for m < M, shift along T with a
 *   zero first row per sequence (model.py:67-75, 188-196, 260-261); mix (M, C);
 *   out (M, rows, C).  C * sizeof(dtype) % 16 == 0.
 * rwkv_tmix_mid (model.py:200-226): with wl = tanh(xw@w1)@w2, al = (xa@a1)@a2,
 *   vl = (xv@v1)@v2 already computed,
 *     w_out = -softplus(-(w0 + wl)) - 0.5                (fp32; w0 fp32)
 *     v_out = v + (v_first - v) * sigmoid(v0 + vl)       (v if layer0)
 *     a     = sigmoid(a0 + al)
 *     kk    = normalize_per_64(k * k_k)                  (eps 1e-12)
 *     k_out = k * (1 + (a - 1) * k_a);  a_out = -kk;  b_out = kk * a
 * rwkv_tmix_post (model.py:229-239): out = (GroupNorm(y) + bonus * v) * g with
 *   GroupNorm over H groups (per_head = 0: MLX's default grouping, channel c in
 *   group c % H; per_head = 1: contiguous groups), weight ln_w, bias ln_b, eps;
 *   bonus per head = sum(r * k * r_k).
 * rwkv_relu_sq: x = relu(x)^2 in place (model.py:262).
 * rwkv_add_layernorm: x_out = x + delta (skipped when delta is NULL);
 *   y = LayerNorm(x_out) with weight w, bias b, eps (model.py:315-326). */
int rwkv_lerp(const void* x, const void* mix, void* out, int M, long long rows, int T, int C,
              int dtype, void* stream);
/* rwkv_lerp_prev: rwkv_lerp whose shift at the first row of sequence s takes
 * prev[s] (rows / T, C) instead of zeros: the RNN-mode token shift with the stored
 * previous token (model.py:449-455, 498-501); prev NULL = rwkv_lerp.                 */
int rwkv_lerp_prev(const void* x, const void* prev, const void* mix, void* out, int M,
                   long long rows, int T, int C, int dtype, void* stream);
/* rwkv_lerp_prev that also stores each sequence's last x row into prev_out (rows / T, C):
 * the token-shift state of an RNN step, written by the same pass that reads the old
 * state.  prev_out may be prev only when T == 1 (decode: each thread reads its vector of
 * the old state before it overwrites it); otherwise RWKV_ERR_ARG. */
int rwkv_lerp_prev_state(const void* x, const void* prev, const void* mix, void* out, void* prev_out, int M,
                         long long rows, int T, int C, int dtype, void* stream);
int rwkv_tmix_mid(const void* k, const void* v, const void* wl, const void* al, const void* vl,
                  const void* v_first, const float* w0, const void* a0, const void* v0,
                  const void* k_k, const void* k_a, float* w_out, void* k_out, void* v_out,
                  void* a_out, void* b_out, long long rows, int C, int layer0, int dtype,
                  void* stream);
int rwkv_tmix_post(const void* y, const void* r, const void* k, const void* v, const void* g,
                   const void* ln_w, const void* ln_b, const void* r_k, void* out, long long rows,
                   int C, int H, float eps, int per_head, int dtype, void* stream);
int rwkv_relu_sq(void* x, long long n, int dtype, void* stream);
/* In place on h (4, n) (the stacked first-stage TimeMix LoRA products v, w, a, g):
 * tanh on h[1], sigmoid on h[3] (model.py:204, :212); h[0], h[2] untouched. */
int rwkv_lora_act(void* h, long long n, int dtype, void* stream);
/* Greedy decoding's next token (the batched decode graph): out[row] = index of the first
 * maximum of x[row, 0:V] (row stride ld), as torch.argmax, in int64. */
int rwkv_argmax_rows(const void* x, long long ld, long long rows, int V, int64_t* out, int dtype, void* stream);
int rwkv_add_layernorm(const void* x, const void* delta, const void* w, const void* b,
                       void* x_out, void* y, long long rows, int C, float eps, int dtype,
                       void* stream);

/* ------------------------------------------------------------------------ */
/* Training loss (l2_wrap_loss / l2_wrap_loss_masked, train.py:317-362) over
 * vocabulary chunks, so that a fused head + loss never holds the full logits.
 *
 * rwkv_ce_chunk: for token i (row i of `logits`, row stride `ld` elements), the
 *   columns [col0, col0 + ncols) of the vocabulary: updates the token's state
 *   float4 {running max m, sum of exp(l - m), target logit, first argmax (int bits)}
 *   (first != 0 starts it).  targets int32 in [0, V); state 16-byte aligned.
 * rwkv_ce_finalize: out fp32[4] = {loss, cross-entropy term, L2 term, denominator}:
 *   loss = sum_i w_i (log s_i + m_i - target logit_i) / den + l2_factor * 0.5 * sum_i m_i^2
 *   with w = mask (den = sum(mask) + 1e-9, train.py:355-356) or 1 (den = ntok).
 *   l2_factor = 1e-4 / (B * T) (train.py:332).
 * rwkv_ce_chunk_grad: d loss / d logits for a chunk times the device scalar *g:
 *   *g * w_i / den * (softmax_ij - [j = target_i]) + *g * l2_factor * m_i * [j = argmax_i]
 *   written to dlogits (row stride ld_out), in dtype; with scaled = 0 the values are
 *   multiplied by den / *g (O(1) entries for 16-bit types; the caller scales the
 *   products it forms from them by *g / den).                                */
/* Fused output head + loss statistics on the tcgen05 tensor cores: for token i,
 * the logits x[i] @ head^T (head (V, K), rounded to dtype as the reference's head
 * output is) are folded into the rwkv_ce_chunk state float4 of all V columns at
 * once inside the GEMM epilogue; no logit is written to memory.  x (M, K) and
 * head in dtype (fp16 / bf16), 16-byte aligned, K % 8 == 0; workspace of
 * rwkv_head_ce_workspace_size(M, V) bytes (16-byte aligned).  Follow with
 * rwkv_ce_finalize.
 * rwkv_head_ce_grad: rwkv_ce_chunk_grad of the vocabulary columns
 * [col0, col0 + ncols) with the logits recomputed from x and the head rows
 * w = head + col0 * K (ncols of them) instead of read from memory. */
size_t rwkv_head_ce_workspace_size(int M, int V);
int rwkv_head_ce_stats(const void* x, const void* head, const int32_t* targets, float* state, int M, int V,
                       int K, void* workspace, size_t workspace_bytes, int dtype, void* stream);
int rwkv_head_ce_grad(const void* x, const void* w, const int32_t* targets, const float* state,
                      const float* mask, const float* out, const float* g, float l2_factor, int scaled,
                      void* dlogits, long long ld_out, int M, int ncols, int K, int col0, int dtype,
                      void* stream);
int rwkv_ce_chunk(const void* logits, long long ld, const int32_t* targets, float* state, int ntok,
                  int col0, int ncols, int first, int dtype, void* stream);
int rwkv_ce_finalize(const float* state, const float* mask, float l2_factor, float* out, int ntok,
                     void* stream);
int rwkv_ce_chunk_grad(const void* logits, long long ld, const int32_t* targets, const float* state,
                       const float* mask, const float* out, const float* g, float l2_factor,
                       int scaled, void* dlogits, long long ld_out, int ntok, int col0, int ncols,
                       int dtype, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* RWKV_B200_H */

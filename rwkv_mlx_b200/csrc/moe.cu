// LoRA-MoE ChannelMix kernels (reference rwkv_mlx/moe.py:35-163).
//
//   moe_router_mma : fp32-accurate logits x @ Wg^T (+ optional bias) on mma.sync for
//                    16-bit x (split gate weights), quad-level top-k (ties -> lower
//                    expert id), softmax over the selected logits, per-CTA partial sums
//                    for aux / z-loss (moe.py:56-84); moe_router: the same on FMAs for
//                    fp32 x.
//   moe_finalize   : deterministic (fixed-order) reduction of those partials.
//   moe_lora_apply : the fused adapter apply on mma.sync (the tcgen05 + TMA kernel that
//                    runs by default is in moe_apply_tc.cu).
//   moe_count / moe_scan / moe_scatter : stable counting sort of the
//                    (token, slot) entries by expert -> perm, inv, offsets.
//   moe_lora_down  : h[p] = x[token(p)] @ A[e(p)]  for every sorted entry p.
//   moe_combine    : out[t] = base[t] + sum_slot score * (h @ B[e]).
//   moe_ortho      : sum_{i<j} ||A_i^T A_j||_F^2 (moe.py:149-163).
#include <cfloat>
#include <type_traits>

#include "common.cuh"

namespace rwkv {

constexpr int ROUTER_WARPS = 8;
constexpr int ROUTER_MAX_CTAS = 148 * 2;  // resident at once: the gate weights are staged once per CTA
constexpr int PERM_TILE = 2048;
constexpr int PERM_THREADS = 256;

__host__ __device__ inline int router_ctas(int ntok) {
    int need = (ntok + ROUTER_WARPS - 1) / ROUTER_WARPS;
    return need < ROUTER_MAX_CTAS ? need : ROUTER_MAX_CTAS;
}

// ---------------------------------------------------------------------------
// Router
// ---------------------------------------------------------------------------
// One warp routes 32 / EM tokens per pass (EM = expert count rounded up to 8, 16 or
// 32): every gate weight read from shared memory serves all of them.  The 32 partial
// logits per lane (token t, expert e at index t * EM + e) are summed over the warp
// by a transpose-reduce (31 shuffles), which leaves lane (t, e) with logit e of
// token t; softmax statistics and top-k then run inside groups of EM lanes.
template <typename T, int EM>
__global__ void __launch_bounds__(ROUTER_WARPS * 32)
    moe_router_kernel(const T* __restrict__ x, const float* __restrict__ gate_w,
                      const float* __restrict__ bias, float* __restrict__ logits,
                      int32_t* __restrict__ inds, T* __restrict__ scores,
                      float* __restrict__ part_f, int32_t* __restrict__ part_c, int ntok, int C,
                      int E, int topk) {
    constexpr int TPW = 32 / EM;
    extern __shared__ __align__(16) float wsm[];  // [E][C] gate weights (two planes per expert)
    __shared__ float red_f[ROUTER_WARPS][EM + 1];
    __shared__ int red_c[ROUTER_WARPS][EM];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // expert e's weights as two planes of C / 2: plane p holds, for each 8-column
    // vector vi, columns 8 vi + 4 p .. 8 vi + 4 p + 3, so that the lanes of a warp
    // (consecutive vi) read consecutive 16-byte words (no bank conflicts)
    if ((reinterpret_cast<uintptr_t>(gate_w) & 15) == 0) {
        for (int i = tid * 4; i < E * C; i += blockDim.x * 4) {
            const int e = i / C, c = i - e * C;
            *reinterpret_cast<float4*>(wsm + e * C + ((c >> 2) & 1) * (C >> 1) + (c >> 3) * 4) =
                *reinterpret_cast<const float4*>(gate_w + i);
        }
    } else {
        for (int i = tid; i < E * C; i += blockDim.x) {
            const int e = i / C, c = i - e * C;
            wsm[e * C + ((c >> 2) & 1) * (C >> 1) + (c >> 3) * 4 + (c & 3)] = gate_w[i];
        }
    }
    __syncthreads();

    const int grp = lane / EM, el = lane % EM;  // token slot of the pass, expert of this lane
    const bool evalid = el < E;
    float acc_p = 0.f, acc_z = 0.f;  // lane (t, e): sum of p_e; lanes e == 0: sum of lse^2
    int acc_c = 0;                   // lane (t, e): count of expert e
    const float lbias = (bias && evalid) ? bias[el] : 0.f;
    const int nvec = C / 8;
    const int stride = gridDim.x * ROUTER_WARPS * TPW;
    for (int tb = (blockIdx.x * ROUTER_WARPS + warp) * TPW; tb < ntok; tb += stride) {
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; i++) v[i] = 0.f;
        for (int vi = lane; vi < nvec; vi += 32) {
            float xf[TPW][8];
#pragma unroll
            for (int t = 0; t < TPW; t++) {
                const int tok = tb + t;
                if (tok < ntok) {
                    const T* xr = x + (size_t)tok * C + vi * 8;
                    if constexpr (sizeof(T) == 2) {
                        const uint4 raw = *reinterpret_cast<const uint4*>(xr);
                        const T* h = reinterpret_cast<const T*>(&raw);
#pragma unroll
                        for (int q = 0; q < 8; q++) xf[t][q] = to_f32(h[q]);
                    } else {
                        const float4 r0 = *reinterpret_cast<const float4*>(xr);
                        const float4 r1 = *reinterpret_cast<const float4*>(xr + 4);
                        xf[t][0] = r0.x, xf[t][1] = r0.y, xf[t][2] = r0.z, xf[t][3] = r0.w;
                        xf[t][4] = r1.x, xf[t][5] = r1.y, xf[t][6] = r1.z, xf[t][7] = r1.w;
                    }
                } else {
#pragma unroll
                    for (int q = 0; q < 8; q++) xf[t][q] = 0.f;
                }
            }
#pragma unroll
            for (int e = 0; e < EM; e++) {
                if (e < E) {
                    const float4 w0 = *reinterpret_cast<const float4*>(wsm + e * C + vi * 4);
                    const float4 w1 = *reinterpret_cast<const float4*>(wsm + e * C + (C >> 1) + vi * 4);
#pragma unroll
                    for (int t = 0; t < TPW; t++) {
                        float a_ = v[t * EM + e];
                        a_ = fmaf(xf[t][0], w0.x, a_), a_ = fmaf(xf[t][1], w0.y, a_);
                        a_ = fmaf(xf[t][2], w0.z, a_), a_ = fmaf(xf[t][3], w0.w, a_);
                        a_ = fmaf(xf[t][4], w1.x, a_), a_ = fmaf(xf[t][5], w1.y, a_);
                        a_ = fmaf(xf[t][6], w1.z, a_), a_ = fmaf(xf[t][7], w1.w, a_);
                        v[t * EM + e] = a_;
                    }
                }
            }
        }
        // transpose-reduce: after the step with offset o a lane keeps the half of its
        // values whose index bit o matches its own lane bit
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            const bool up = lane & o;
#pragma unroll
            for (int i = 0; i < o; i++) {
                const float send = up ? v[i] : v[i + o];
                const float keep = up ? v[i + o] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
        }
        const int tok = tb + grp;
        const bool tvalid = tok < ntok, valid = evalid && tvalid;
        const float lg = evalid ? v[0] + lbias : -INFINITY;
        if (logits && valid) logits[(size_t)tok * E + el] = lg;

        // full softmax statistics (max-stabilised log-sum-exp) within the group
        float m = lg;
#pragma unroll
        for (int o = EM / 2; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float ex = evalid ? expf(lg - m) : 0.f;
        float se = ex;
#pragma unroll
        for (int o = EM / 2; o > 0; o >>= 1) se += __shfl_xor_sync(0xffffffffu, se, o);
        if (valid) acc_p += ex / se;
        const float lse = m + logf(se);
        if (el == 0 && tvalid) acc_z = fmaf(lse, lse, acc_z);

        // top-k by repeated argmax, ties to the lower expert id
        bool taken = !evalid;
        float sel0 = 0.f, denom = 0.f, my_sel_logit = 0.f;
        int my_slot = -1;
        for (int kk = 0; kk < topk; kk++) {
            float bv = taken ? -INFINITY : lg;
            int bi = taken ? 0x7fffffff : el;
#pragma unroll
            for (int o = EM / 2; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) bv = ov, bi = oi;
            }
            if (kk == 0) sel0 = bv;
            denom += expf(bv - sel0);
            if (el == bi) {
                taken = true;
                my_slot = kk;
                my_sel_logit = bv;
            }
            if (el == 0 && tvalid) inds[(size_t)tok * topk + kk] = bi;
        }
        if (my_slot >= 0 && tvalid) {
            scores[(size_t)tok * topk + my_slot] = from_f32<T>(expf(my_sel_logit - sel0) / denom);
            acc_c += 1;
        }
    }
    // sum over the token slots of the warp (lanes with the same expert)
#pragma unroll
    for (int o = EM; o < 32; o <<= 1) {
        acc_p += __shfl_xor_sync(0xffffffffu, acc_p, o);
        acc_c += __shfl_xor_sync(0xffffffffu, acc_c, o);
        acc_z += __shfl_xor_sync(0xffffffffu, acc_z, o);
    }
    if (lane < EM) {
        red_f[warp][lane] = evalid ? acc_p : 0.f;
        red_c[warp][lane] = evalid ? acc_c : 0;
    }
    if (lane == 0) red_f[warp][EM] = acc_z;
    __syncthreads();
    if (tid < E) {
        float s_ = 0.f;
        int c = 0;
        for (int w = 0; w < ROUTER_WARPS; w++) s_ += red_f[w][tid], c += red_c[w][tid];
        part_f[(size_t)blockIdx.x * (E + 1) + tid] = s_;
        part_c[(size_t)blockIdx.x * E + tid] = c;
    }
    if (tid == 0) {
        float s_ = 0.f;
        for (int w = 0; w < ROUTER_WARPS; w++) s_ += red_f[w][EM];
        part_f[(size_t)blockIdx.x * (E + 1) + E] = s_;
    }
}

// Fixed-order (deterministic) reduction of the per-CTA partials: thread t sums CTAs
// t, t + 256, ..., then warps and finally 8 warp totals, always in the same order.
constexpr int FIN_THREADS = 256;
template <int FIN_MAXE>  // expert count rounded up to 8, 16 or 32
__global__ void __launch_bounds__(FIN_THREADS)
    moe_router_finalize_kernel(const float* __restrict__ part_f, const int32_t* __restrict__ part_c,
                               int nblk, int ntok, int E, int topk, float* __restrict__ stats,
                               int32_t* __restrict__ counts) {
    __shared__ float wf[FIN_THREADS / 32][FIN_MAXE + 1];
    __shared__ int wc[FIN_THREADS / 32][FIN_MAXE];
    __shared__ float fp[FIN_MAXE];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float p[FIN_MAXE + 1];
    int c[FIN_MAXE];
#pragma unroll
    for (int q = 0; q <= FIN_MAXE; q++) p[q] = 0.f;
#pragma unroll
    for (int q = 0; q < FIN_MAXE; q++) c[q] = 0;
    for (int b = tid; b < nblk; b += FIN_THREADS) {
#pragma unroll
        for (int q = 0; q <= FIN_MAXE; q++)
            if (q <= E) p[q] += part_f[(size_t)b * (E + 1) + q];
#pragma unroll
        for (int q = 0; q < FIN_MAXE; q++)
            if (q < E) c[q] += part_c[(size_t)b * E + q];
    }
#pragma unroll
    for (int q = 0; q <= FIN_MAXE; q++) {
        if (q <= E) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) p[q] += __shfl_xor_sync(0xffffffffu, p[q], o);
            if (lane == 0) wf[warp][q] = p[q];
        }
    }
#pragma unroll
    for (int q = 0; q < FIN_MAXE; q++) {
        if (q < E) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) c[q] += __shfl_xor_sync(0xffffffffu, c[q], o);
            if (lane == 0) wc[warp][q] = c[q];
        }
    }
    __syncthreads();
    if (tid <= E) {
        float sp = 0.f;
        long long sc = 0;
        for (int w = 0; w < FIN_THREADS / 32; w++) {
            sp += wf[w][tid];
            if (tid < E) sc += wc[w][tid];
        }
        if (tid < E) {
            const float pe = sp / (float)ntok;
            const float fe = (float)sc / ((float)ntok * (float)topk);
            stats[2 + tid] = fe;
            fp[tid] = fe * pe;
            if (counts) counts[tid] = (int32_t)sc;
        } else {
            stats[1] = sp / (float)ntok;
        }
    }
    __syncthreads();
    if (tid == 0) {
        float aux = 0.f;
        for (int i = 0; i < E; i++) aux += fp[i];
        stats[0] = (float)E * aux;
    }
}

// ---------------------------------------------------------------------------
// Permutation (stable counting sort by expert)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(PERM_THREADS)
    moe_count_kernel(const int32_t* __restrict__ inds, int n, int E, int32_t* __restrict__ blkcnt) {
    extern __shared__ int hist[];
    for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
    __syncthreads();
    const int t0 = blockIdx.x * PERM_TILE;
    const int t1 = min(n, t0 + PERM_TILE);
    for (int i = t0 + threadIdx.x; i < t1; i += blockDim.x) atomicAdd(&hist[inds[i]], 1);
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) blkcnt[(size_t)blockIdx.x * E + e] = hist[e];
}

// blkoff[b][e] = start of expert e + entries of e in tiles < b ; offsets[E+1]
__global__ void moe_scan_kernel(const int32_t* __restrict__ blkcnt, int nblk, int E,
                                int32_t* __restrict__ blkoff, int32_t* __restrict__ offsets) {
    extern __shared__ int tot[];
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int s = 0;
        for (int b = 0; b < nblk; b++) {
            blkoff[(size_t)b * E + e] = s;
            s += blkcnt[(size_t)b * E + e];
        }
        tot[e] = s;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int s = 0;
        for (int e = 0; e < E; e++) {
            offsets[e] = s;
            const int t = tot[e];
            tot[e] = s;
            s += t;
        }
        offsets[E] = s;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        const int st = tot[e];
        for (int b = 0; b < nblk; b++) blkoff[(size_t)b * E + e] += st;
    }
}

__global__ void __launch_bounds__(PERM_THREADS)
    moe_scatter_kernel(const int32_t* __restrict__ inds, int n, int E,
                       const int32_t* __restrict__ blkoff, int32_t* __restrict__ perm,
                       int32_t* __restrict__ inv) {
    constexpr int NW = PERM_THREADS / 32, SUB = PERM_TILE / NW;
    extern __shared__ int sm[];
    int* wcnt = sm;           // [NW][E]
    int* wrun = sm + NW * E;  // [NW][E]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < NW * E; i += blockDim.x) wcnt[i] = 0;
    __syncthreads();
    const int s0 = blockIdx.x * PERM_TILE + warp * SUB;
    const int s1 = min(n, s0 + SUB);
    for (int i = s0 + lane; i < s1; i += 32) atomicAdd(&wcnt[warp * E + inds[i]], 1);
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int s = blkoff[(size_t)blockIdx.x * E + e];
        for (int w = 0; w < NW; w++) {
            wrun[w * E + e] = s;
            s += wcnt[w * E + e];
        }
    }
    __syncthreads();
    for (int base = s0; base < s1; base += 32) {
        const int i = base + lane;
        const bool act = i < s1;
        const unsigned mask = __ballot_sync(0xffffffffu, act);
        if (act) {
            const int e = inds[i];
            const unsigned peers = __match_any_sync(mask, e);
            const int rank = __popc(peers & ((1u << lane) - 1u));
            const int pos = wrun[warp * E + e] + rank;
            perm[pos] = i;
            inv[i] = pos;
            __syncwarp(mask);
            if (rank == 0) wrun[warp * E + e] += __popc(peers);
        }
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------
// Grouped LoRA down-projection: one warp per sorted entry.
// ---------------------------------------------------------------------------
template <typename T, int R>
__global__ void __launch_bounds__(256)
    moe_lora_down_kernel(const T* __restrict__ x, const T* __restrict__ A,
                         const int32_t* __restrict__ perm, const int32_t* __restrict__ offsets,
                         float* __restrict__ h, int n, int C, int E, int topk) {
    __shared__ int offs[257];
    for (int i = threadIdx.x; i <= E; i += blockDim.x) offs[i] = offsets[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int p = blockIdx.x * 8 + warp; p < n; p += gridDim.x * 8) {
        int e = 0;
        while (e + 1 < E && offs[e + 1] <= p) e++;
        const int tok = perm[p] / topk;
        const T* xr = x + (size_t)tok * C;
        const T* Ae = A + (size_t)e * C * R;
        float acc[R];
#pragma unroll
        for (int q = 0; q < R; q++) acc[q] = 0.f;
        for (int c = lane; c < C; c += 32) {
            const float xv = to_f32(xr[c]);
            const T* ar = Ae + (size_t)c * R;
#pragma unroll
            for (int q = 0; q < R; q++) acc[q] = fmaf(xv, to_f32(ar[q]), acc[q]);
        }
#pragma unroll
        for (int q = 0; q < R; q++) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[q] += __shfl_xor_sync(0xffffffffu, acc[q], o);
        }
        if (lane == 0) {
#pragma unroll
            for (int q = 0; q < R; q++) h[(size_t)p * R + q] = acc[q];
        }
    }
}

// ---------------------------------------------------------------------------
// Combine: one warp per token.
// ---------------------------------------------------------------------------
template <typename T, int R>
__global__ void __launch_bounds__(256)
    moe_combine_kernel(const T* base, const float* __restrict__ h, const T* __restrict__ B,
                       const int32_t* __restrict__ inds, const T* __restrict__ scores,
                       const int32_t* __restrict__ inv, T* out, int ntok, int C, int topk) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int tok = blockIdx.x * 8 + warp; tok < ntok; tok += gridDim.x * 8) {
        float hs[8][R];  // topk <= 8
        int es[8];
        for (int s = 0; s < topk; s++) {
            const int ent = tok * topk + s;
            const int p = inv[ent];
            es[s] = inds[ent];
            const float sc = to_f32(scores[ent]);
#pragma unroll
            for (int q = 0; q < R; q++) hs[s][q] = sc * h[(size_t)p * R + q];
        }
        for (int c = lane; c < C; c += 32) {
            float o = base ? to_f32(base[(size_t)tok * C + c]) : 0.f;
            for (int s = 0; s < topk; s++) {
                const T* Be = B + (size_t)es[s] * R * C + c;
                float d = 0.f;
#pragma unroll
                for (int q = 0; q < R; q++) d = fmaf(hs[s][q], to_f32(Be[(size_t)q * C]), d);
                o += d;
            }
            out[(size_t)tok * C + c] = from_f32<T>(o);
        }
    }
}

// ---------------------------------------------------------------------------
// Orthogonality loss, one CTA; thread (r1, r2) accumulates every pair i<j.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(1024)
    moe_ortho_kernel(const T* __restrict__ A, float* __restrict__ out, int E, int C, int R) {
    __shared__ float red[32];
    float tot = 0.f;
    for (int idx = threadIdx.x; idx < R * R; idx += blockDim.x) {
        const int r1 = idx / R, r2 = idx % R;
        for (int i = 0; i < E; i++)
            for (int j = i + 1; j < E; j++) {
                const T* Ai = A + (size_t)i * C * R;
                const T* Aj = A + (size_t)j * C * R;
                float s = 0.f;
                for (int c = 0; c < C; c++) s = fmaf(to_f32(Ai[(size_t)c * R + r1]), to_f32(Aj[(size_t)c * R + r2]), s);
                tot = fmaf(s, s, tot);
            }
    }
    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = tot;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.f;
        for (int w = 0; w < (int)(blockDim.x + 31) / 32; w++) s += red[w];
        *out = s;
    }
}

// ---------------------------------------------------------------------------
// Expert-parallel helpers: dispatch gather, per-entry up-projection, combine of rows.
// ---------------------------------------------------------------------------
// rows[p] = x[perm[p] / topk]; one warp per row, 16-byte vectors.
template <typename T>
__global__ void __launch_bounds__(256)
    moe_gather_rows_kernel(const T* __restrict__ x, const int32_t* __restrict__ perm,
                           T* __restrict__ rows, int n, int C, int topk) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nv = C * (int)sizeof(T) / 16;
    for (int p = blockIdx.x * 8 + warp; p < n; p += gridDim.x * 8) {
        const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(perm[p] / topk) * C);
        uint4* dst = reinterpret_cast<uint4*>(rows + (size_t)p * C);
        for (int i = lane; i < nv; i += 32) dst[i] = src[i];
    }
}

// Full-expert dispatch (MoE_CMix, moe.py:231-236): for sorted position p with
// tok = perm[p] / topk and expert e(p) (from offsets),
//   rows[p] = x[tok] + (x_prev(tok) - x[tok]) * x_k[e(p)]
// where x_prev(tok) is the previous token of the same sequence (sequences of T tokens),
// or prev[tok / T] (NULL: zeros) for the first token.  One warp per row, one 16-byte
// vector per lane step; fp32 arithmetic, one rounding.
template <typename T>
__global__ void __launch_bounds__(256)
    moe_expert_mix_rows_kernel(const T* __restrict__ x, const T* __restrict__ prev, const T* __restrict__ x_k,
                               const int32_t* __restrict__ perm, const int32_t* __restrict__ offsets,
                               T* __restrict__ rows, int n, int T_, int C, int topk, int E) {
    constexpr int V = 16 / sizeof(T);
    __shared__ int offs[257];
    for (int i = threadIdx.x; i <= E; i += blockDim.x) offs[i] = offsets[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nv = C / V;
    for (int p = blockIdx.x * 8 + warp; p < n; p += gridDim.x * 8) {
        int e = 0;
        while (e + 1 < E && offs[e + 1] <= p) e++;
        const int tok = perm[p] / topk;
        const T* xr = x + (size_t)tok * C;
        const T* pr = (tok % T_) ? xr - C : (prev ? prev + (size_t)(tok / T_) * C : nullptr);
        const T* mr = x_k + (size_t)e * C;
        T* out = rows + (size_t)p * C;
        for (int i = lane; i < nv; i += 32) {
            const uint4 xv = reinterpret_cast<const uint4*>(xr)[i];
            const uint4 mv = reinterpret_cast<const uint4*>(mr)[i];
            uint4 pv = make_uint4(0, 0, 0, 0);
            if (pr) pv = reinterpret_cast<const uint4*>(pr)[i];
            const T* xe = reinterpret_cast<const T*>(&xv);
            const T* me = reinterpret_cast<const T*>(&mv);
            const T* pe = reinterpret_cast<const T*>(&pv);
            uint4 ov;
            T* oe = reinterpret_cast<T*>(&ov);
#pragma unroll
            for (int q = 0; q < V; q++) {
                const float xf = to_f32(xe[q]);
                oe[q] = from_f32<T>(fmaf(to_f32(pe[q]) - xf, to_f32(me[q]), xf));
            }
            reinterpret_cast<uint4*>(out)[i] = ov;
        }
    }
}

// y[dst(p)] = h[p] @ B[e(p)], e(p) from offsets, dst(p) = out_index ? out_index[p] : p.
template <typename T, int R>
__global__ void __launch_bounds__(256)
    moe_lora_up_kernel(const float* __restrict__ h, const T* __restrict__ B,
                       const int32_t* __restrict__ offsets, const int32_t* __restrict__ out_index,
                       T* __restrict__ y, int n, int C, int E) {
    __shared__ int offs[257];
    for (int i = threadIdx.x; i <= E; i += blockDim.x) offs[i] = offsets[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int p = blockIdx.x * 8 + warp; p < n; p += gridDim.x * 8) {
        int e = 0;
        while (e + 1 < E && offs[e + 1] <= p) e++;
        float hv[R];
#pragma unroll
        for (int q = 0; q < R; q++) hv[q] = h[(size_t)p * R + q];
        const T* Be = B + (size_t)e * R * C;
        T* out = y + (size_t)(out_index ? out_index[p] : p) * C;
        for (int c = lane; c < C; c += 32) {
            float d = 0.f;
#pragma unroll
            for (int q = 0; q < R; q++) d = fmaf(hv[q], to_f32(Be[(size_t)q * C + c]), d);
            out[c] = from_f32<T>(d);
        }
    }
}

// out[t] = base[t] + sum_s scores[t, s] * rows[inv[t * topk + s]]; one warp per token,
// one 16-byte vector per lane step when every row is 16-byte aligned (vec), else scalar.
template <typename T>
__global__ void __launch_bounds__(256)
    moe_combine_rows_kernel(const T* base, const T* __restrict__ rows, const T* __restrict__ scores,
                            const int32_t* __restrict__ inv, T* out, int ntok, int C, int topk, int vec) {
    constexpr int V = 16 / sizeof(T);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int t = blockIdx.x * 8 + warp; t < ntok; t += gridDim.x * 8) {
        if (vec) {
            for (int i = lane; i < C / V; i += 32) {
                float o[V];
                if (base) {
                    const uint4 bv = reinterpret_cast<const uint4*>(base + (size_t)t * C)[i];
                    const T* be = reinterpret_cast<const T*>(&bv);
#pragma unroll
                    for (int q = 0; q < V; q++) o[q] = to_f32(be[q]);
                } else {
#pragma unroll
                    for (int q = 0; q < V; q++) o[q] = 0.f;
                }
                for (int s = 0; s < topk; s++) {
                    const int ent = t * topk + s;
                    const float sc = to_f32(scores[ent]);
                    const uint4 rv = reinterpret_cast<const uint4*>(rows + (size_t)inv[ent] * C)[i];
                    const T* re = reinterpret_cast<const T*>(&rv);
#pragma unroll
                    for (int q = 0; q < V; q++) o[q] = fmaf(sc, to_f32(re[q]), o[q]);
                }
                uint4 ov;
                T* oe = reinterpret_cast<T*>(&ov);
#pragma unroll
                for (int q = 0; q < V; q++) oe[q] = from_f32<T>(o[q]);
                reinterpret_cast<uint4*>(out + (size_t)t * C)[i] = ov;
            }
        } else {
            for (int c = lane; c < C; c += 32) {
                float o = base ? to_f32(base[(size_t)t * C + c]) : 0.f;
                for (int s = 0; s < topk; s++) {
                    const int ent = t * topk + s;
                    o = fmaf(to_f32(scores[ent]), to_f32(rows[(size_t)inv[ent] * C + c]), o);
                }
                out[(size_t)t * C + c] = from_f32<T>(o);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Fused adapter apply (tensor cores):  out[t] = base[t] + sum_s scores[t,s] * (x[t] @ A[e]) @ B[e]
// with e = inds[t,s].  Per tile of 64 tokens (4 warps x 16), dense over all E*R adapter
// columns on mma.sync m16n8k16 (fp32 accumulate): H = X @ [A_0 | ... | A_E-1] in
// K-slices of 64 channels, H masked and scaled by the routing scores (0 for experts a
// token did not select, as in the reference's dense sum), then OUT = base + H @ [B_0; ...]
// in N-slices of 64 channels.  H goes from the accumulators straight into the A
// fragments of the second product (rounded to the activation dtype).  x and base are
// read once and nothing per entry goes through global memory.  Weight slices are
// staged with cp.async in their natural layouts and read with ldmatrix(.trans).
// ---------------------------------------------------------------------------
namespace apply {
constexpr int TM = 64, KS = 64, NTH = 128;
__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void cp16(void* dst, const void* src, bool ok) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(su32(dst)), "l"(src), "r"(ok ? 16 : 0) : "memory");
}
__device__ __forceinline__ void ldm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(su32(p)));
}
__device__ __forceinline__ void ldm_x4_t(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(su32(p)));
}
template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    if constexpr (std::is_same<T, __half>::value)
        asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                     : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    else
        asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                     : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    T h[2] = {from_f32<T>(lo), from_f32<T>(hi)};
    return *reinterpret_cast<uint32_t*>(h);
}
template <int EN>
struct Geo {
    static constexpr int XP = KS * 2 + 16;  // X slice row pitch (bytes): TM rows x KS channels
    static constexpr int AP = EN * 2 + 16;  // A slice row pitch: KS channels x EN columns
    static constexpr int BP = KS * 2 + 16;  // B slice row pitch: EN rows x KS channels
    static constexpr int OP = KS * 2 + 16;  // base / out slice row pitch: TM rows x KS channels
    static constexpr int XS = TM * XP, AS = KS * AP, BS = EN * BP, OS = TM * OP;
    static constexpr int STAGE = (XS + AS) > (BS + OS) ? (XS + AS) : (BS + OS);
    static constexpr int SMEM = 2 * STAGE;
};
}  // namespace apply

// Router on the tensor cores for 16-bit x (mma.sync m16n8k16, fp32 accumulate; the GEMM
// is 16 tokens x E experts x C per warp and memory-bound, so the legacy MMA suffices).
// The fp32 gate weights are split into 16-bit terms W = W0 + W1 / S + W2 / S^2 (S = 2^11
// and two terms for fp16, S = 2^8 and three terms for bf16), each term with its own fp32
// accumulator: x is exact in its own type and every 16-bit x 16-bit product is exact in
// fp32, so the logits carry fp32-level rounding like the FMA kernel's.  Within every
// 32-column block the K order is permuted identically for x and W (the fragment slots of
// thread t of a quad are columns 8t .. 8t+7), so each operand load is one 16-byte vector.
// Thread (g, t) of a warp holds the logits of tokens g and g + 8 of its 16 for experts
// 8n + 2t and 8n + 2t + 1; softmax statistics and top-k (ties to the lower expert id) run
// over the quad.
__host__ __device__ inline int router_mma_rs(int C) {  // W row stride (elements): 64 B mod 128 B
    return (((C * 2 + 127) / 128) * 128 + 64) / 2;
}
template <typename T>
__host__ __device__ constexpr int router_mma_terms() { return sizeof(T) == 2 && !std::is_same<T, __nv_bfloat16>::value ? 2 : 3; }

template <typename T, int NT>
__global__ void __launch_bounds__(ROUTER_WARPS * 32)
    moe_router_mma_kernel(const T* __restrict__ x, const float* __restrict__ gate_w,
                          const float* __restrict__ bias, float* __restrict__ logits,
                          int32_t* __restrict__ inds, T* __restrict__ scores, float* __restrict__ part_f,
                          int32_t* __restrict__ part_c, int ntok, int C, int E, int topk) {
    constexpr int NTERM = router_mma_terms<T>();
    constexpr float SC = NTERM == 2 ? 2048.f : 256.f;
    constexpr int EM = NT * 8, NO = 2 * NT;  // padded experts; experts owned per thread
    extern __shared__ __align__(16) unsigned char wsm_raw[];
    T* wsm = reinterpret_cast<T*>(wsm_raw);  // [NTERM][EM][RS]
    __shared__ float red_f[ROUTER_WARPS][EM + 1];
    __shared__ int red_c[ROUTER_WARPS][EM];
    const int RS = router_mma_rs(C), CP = RS;  // columns past C are zero
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    // split weights, 4 columns per step (C % 8 == 0: a group of 4 is all in or all out)
    const bool al16 = (reinterpret_cast<uintptr_t>(gate_w) & 15) == 0;
    const int cq = CP / 4;
#pragma unroll 4
    for (int i = tid; i < EM * cq; i += blockDim.x) {
        const int e = i / cq, c = 4 * (i - e * cq);
        float w[4] = {0.f, 0.f, 0.f, 0.f};
        if (e < E && c < C) {
            const float* src = gate_w + (size_t)e * C + c;
            if (al16) {
                const float4 v = __ldg(reinterpret_cast<const float4*>(src));
                w[0] = v.x, w[1] = v.y, w[2] = v.z, w[3] = v.w;
            } else {
                w[0] = src[0], w[1] = src[1], w[2] = src[2], w[3] = src[3];
            }
        }
        T t0[4], t1[4], t2[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            t0[u] = from_f32<T>(w[u]);
            const float r1 = (w[u] - to_f32(t0[u])) * SC;  // exact: t0 is w rounded
            t1[u] = from_f32<T>(r1);
            t2[u] = from_f32<T>((r1 - to_f32(t1[u])) * SC);
        }
        *reinterpret_cast<uint2*>(wsm + (size_t)e * RS + c) = *reinterpret_cast<const uint2*>(t0);
        *reinterpret_cast<uint2*>(wsm + (size_t)(EM + e) * RS + c) = *reinterpret_cast<const uint2*>(t1);
        if constexpr (NTERM == 3)
            *reinterpret_cast<uint2*>(wsm + (size_t)(2 * EM + e) * RS + c) = *reinterpret_cast<const uint2*>(t2);
    }
    __syncthreads();

    float acc_p[NO], acc_z = 0.f;
    int acc_c[NO];
    float lb[NO];
#pragma unroll
    for (int o = 0; o < NO; o++) {
        const int e = 8 * (o >> 1) + 2 * t + (o & 1);
        acc_p[o] = 0.f, acc_c[o] = 0;
        lb[o] = (bias && e < E) ? bias[e] : 0.f;
    }
    const int stride = gridDim.x * ROUTER_WARPS * 16;
    for (int tb = (blockIdx.x * ROUTER_WARPS + warp) * 16; tb < ntok; tb += stride) {
        float d[NTERM][NT][4];
#pragma unroll
        for (int m = 0; m < NTERM; m++)
#pragma unroll
            for (int n = 0; n < NT; n++) d[m][n][0] = d[m][n][1] = d[m][n][2] = d[m][n][3] = 0.f;
        const int r0 = tb + g, r1 = tb + g + 8;
        const T* x0 = x + (size_t)(r0 < ntok ? r0 : 0) * C;
        const T* x1 = x + (size_t)(r1 < ntok ? r1 : 0) * C;
        constexpr int KB = 8;  // 32-column blocks whose x is loaded as one batch (16 loads in flight)
        for (int kb0 = 0; kb0 < C; kb0 += 32 * KB) {
            uint4 a_lo[KB], a_hi[KB];
#pragma unroll
            for (int u = 0; u < KB; u++) {
                const int col = kb0 + 32 * u + 8 * t;
                const bool in = col < C;  // C % 8 == 0: a 16-byte piece is all in or all out
                const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
                a_lo[u] = (in && r0 < ntok) ? __ldg(reinterpret_cast<const uint4*>(x0 + col)) : z4;
                a_hi[u] = (in && r1 < ntok) ? __ldg(reinterpret_cast<const uint4*>(x1 + col)) : z4;
            }
#pragma unroll
            for (int u = 0; u < KB; u++) {
                const int col = kb0 + 32 * u + 8 * t;
                if (kb0 + 32 * u >= C) break;
                const uint32_t A0[4] = {a_lo[u].x, a_hi[u].x, a_lo[u].y, a_hi[u].y};  // columns 8t .. 8t+3
                const uint32_t A1[4] = {a_lo[u].z, a_hi[u].z, a_lo[u].w, a_hi[u].w};  // columns 8t+4 .. 8t+7
#pragma unroll
                for (int m = 0; m < NTERM; m++)
#pragma unroll
                    for (int n = 0; n < NT; n++) {
                        const uint4 b = *reinterpret_cast<const uint4*>(wsm + (size_t)(m * EM + 8 * n + g) * RS + col);
                        apply::mma16816<T>(d[m][n], A0, b.x, b.y);
                        apply::mma16816<T>(d[m][n], A1, b.z, b.w);
                    }
            }
        }
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int tok = tb + g + 8 * h;
            const bool tvalid = tok < ntok;
            float lg[NO];
            bool ev[NO];
#pragma unroll
            for (int o = 0; o < NO; o++) {
                const int n = o >> 1, i = o & 1, e = 8 * n + 2 * t + i;
                float v = d[NTERM - 1][n][2 * h + i];
#pragma unroll
                for (int m = NTERM - 2; m >= 0; m--) v = d[m][n][2 * h + i] + v * (1.f / SC);
                ev[o] = e < E;
                lg[o] = ev[o] ? v + lb[o] : -INFINITY;
                if (logits && tvalid && ev[o]) logits[(size_t)tok * E + e] = lg[o];
            }
            // full softmax statistics (max-stabilised log-sum-exp) over the quad
            float m = -INFINITY;
#pragma unroll
            for (int o = 0; o < NO; o++) m = fmaxf(m, lg[o]);
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
            float ex[NO], se = 0.f;
#pragma unroll
            for (int o = 0; o < NO; o++) ex[o] = ev[o] ? expf(lg[o] - m) : 0.f, se += ex[o];
            se += __shfl_xor_sync(0xffffffffu, se, 1);
            se += __shfl_xor_sync(0xffffffffu, se, 2);
            if (tvalid) {
#pragma unroll
                for (int o = 0; o < NO; o++) acc_p[o] += ev[o] ? ex[o] / se : 0.f;
            }
            const float lse = m + logf(se);
            if (t == 0 && tvalid) acc_z = fmaf(lse, lse, acc_z);

            // top-k by repeated argmax over the quad, ties to the lower expert id
            bool taken[NO];
            int slot[NO];
#pragma unroll
            for (int o = 0; o < NO; o++) taken[o] = !ev[o], slot[o] = -1;
            float sel0 = 0.f, denom = 0.f;
            for (int kk = 0; kk < topk; kk++) {
                float bv = -INFINITY;
                int bi = 0x7fffffff;
#pragma unroll
                for (int o = 0; o < NO; o++) {
                    const int e = 8 * (o >> 1) + 2 * t + (o & 1);
                    if (!taken[o] && (lg[o] > bv || (lg[o] == bv && e < bi))) bv = lg[o], bi = e;
                }
#pragma unroll
                for (int s = 1; s <= 2; s <<= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, s);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, s);
                    if (ov > bv || (ov == bv && oi < bi)) bv = ov, bi = oi;
                }
                if (kk == 0) sel0 = bv;
                denom += expf(bv - sel0);
#pragma unroll
                for (int o = 0; o < NO; o++)
                    if (8 * (o >> 1) + 2 * t + (o & 1) == bi) taken[o] = true, slot[o] = kk;
                if (t == 0 && tvalid) inds[(size_t)tok * topk + kk] = bi;
            }
            if (tvalid) {
#pragma unroll
                for (int o = 0; o < NO; o++)
                    if (slot[o] >= 0) {
                        scores[(size_t)tok * topk + slot[o]] = from_f32<T>(expf(lg[o] - sel0) / denom);
                        acc_c[o] += 1;
                    }
            }
        }
    }
    // per expert over the 8 token groups of the warp, then over the warps of the CTA
#pragma unroll
    for (int s = 4; s < 32; s <<= 1) {
#pragma unroll
        for (int o = 0; o < NO; o++) {
            acc_p[o] += __shfl_xor_sync(0xffffffffu, acc_p[o], s);
            acc_c[o] += __shfl_xor_sync(0xffffffffu, acc_c[o], s);
        }
    }
#pragma unroll
    for (int s = 1; s < 32; s <<= 1) acc_z += __shfl_xor_sync(0xffffffffu, acc_z, s);
    if (g == 0) {
#pragma unroll
        for (int o = 0; o < NO; o++) {
            const int e = 8 * (o >> 1) + 2 * t + (o & 1);
            red_f[warp][e] = acc_p[o];
            red_c[warp][e] = acc_c[o];
        }
    }
    if (lane == 0) red_f[warp][EM] = acc_z;
    __syncthreads();
    if (tid < E) {
        float s_ = 0.f;
        int c = 0;
        for (int w = 0; w < ROUTER_WARPS; w++) s_ += red_f[w][tid], c += red_c[w][tid];
        part_f[(size_t)blockIdx.x * (E + 1) + tid] = s_;
        part_c[(size_t)blockIdx.x * E + tid] = c;
    }
    if (tid == 0) {
        float s_ = 0.f;
        for (int w = 0; w < ROUTER_WARPS; w++) s_ += red_f[w][EM];
        part_f[(size_t)blockIdx.x * (E + 1) + E] = s_;
    }
}


template <typename T, int EN>
__global__ void __launch_bounds__(apply::NTH)
    moe_lora_apply_kernel(const T* __restrict__ x, const T* __restrict__ base, const T* __restrict__ A,
                          const T* __restrict__ B, const int32_t* __restrict__ inds,
                          const T* __restrict__ scores, T* __restrict__ out, int ntok, int C, int R, int E,
                          int topk) {
    using namespace apply;
    using G = Geo<EN>;
    extern __shared__ __align__(16) unsigned char smem_apply[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tg = lane & 3;
    const int t0 = blockIdx.x * TM;
    const int nsl = C / KS;
    const int RP = R / 8;  // 16-byte pieces per adapter row

    auto load_down = [&](int sl, int buf) {
        unsigned char* xs = smem_apply + buf * G::STAGE;
        unsigned char* as = xs + G::XS;
        const int c0 = sl * KS;
        for (int p = tid; p < TM * (KS / 8); p += NTH) {
            const int row = p / (KS / 8), pc = p % (KS / 8), tok = t0 + row;
            const bool ok = tok < ntok;
            cp16(xs + row * G::XP + pc * 16, x + (size_t)(ok ? tok : 0) * C + c0 + pc * 8, ok);
        }
        for (int p = tid; p < E * KS * RP; p += NTH) {
            const int e = p / (KS * RP), rem = p % (KS * RP), c = rem / RP, qp = rem % RP;
            cp16(as + c * G::AP + (e * R + qp * 8) * 2, A + ((size_t)e * C + c0 + c) * R + qp * 8, true);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    auto load_up = [&](int sl, int buf) {
        unsigned char* bs = smem_apply + buf * G::STAGE;
        unsigned char* os = bs + G::BS;
        const int c0 = sl * KS;
        for (int p = tid; p < EN * (KS / 8); p += NTH) {
            const int row = p / (KS / 8), pc = p % (KS / 8);
            cp16(bs + row * G::BP + pc * 16, B + (size_t)row * C + c0 + pc * 8, true);
        }
        for (int p = tid; p < TM * (KS / 8); p += NTH) {  // base slice (zeros when there is no base)
            const int row = p / (KS / 8), pc = p % (KS / 8), tok = t0 + row;
            const bool ok = base && tok < ntok;
            cp16(os + row * G::OP + pc * 16, ok ? base + (size_t)tok * C + c0 + pc * 8 : x, ok);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    // ---- H = X @ Acat ----
    float acc[EN / 8][4];
#pragma unroll
    for (int i = 0; i < EN / 8; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    load_down(0, 0);
    for (int sl = 0; sl < nsl; sl++) {
        if (sl + 1 < nsl) {
            load_down(sl + 1, (sl + 1) & 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const unsigned char* xs = smem_apply + (sl & 1) * G::STAGE;
        const unsigned char* as = xs + G::XS;
#pragma unroll
        for (int kk = 0; kk < KS / 16; kk++) {
            uint32_t af[4];
            ldm_x4(af, xs + (16 * warp + (lane & 15)) * G::XP + (kk * 16 + (lane >> 4) * 8) * 2);
#pragma unroll
            for (int n2 = 0; n2 < EN / 16; n2++) {
                uint32_t bq[4];
                ldm_x4_t(bq, as + (kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * G::AP + (n2 * 16 + (lane >> 4) * 8) * 2);
                mma16816<T>(acc[2 * n2], af, bq[0], bq[1]);
                mma16816<T>(acc[2 * n2 + 1], af, bq[2], bq[3]);
            }
        }
        __syncthreads();
    }
    load_up(0, 0);  // overlaps the routing mask below

    // ---- routing mask / scores: column n belongs to expert n / R ----
#pragma unroll
    for (int hr = 0; hr < 2; hr++) {
        const int tok = t0 + 16 * warp + g + 8 * hr;
        int es[8];
        float ss[8];
        const int kq = tok < ntok ? topk : 0;
        for (int s = 0; s < 8; s++) {
            es[s] = s < kq ? inds[(size_t)tok * topk + s] : -1;
            ss[s] = s < kq ? (scores ? to_f32(scores[(size_t)tok * topk + s]) : 1.f) : 0.f;
        }
#pragma unroll
        for (int nt = 0; nt < EN / 8; nt++) {
            const int e = (nt * 8) / R;
            float gsc = 0.f;
#pragma unroll
            for (int s = 0; s < 8; s++) gsc += es[s] == e ? ss[s] : 0.f;
            acc[nt][2 * hr] *= gsc;
            acc[nt][2 * hr + 1] *= gsc;
        }
    }
    uint32_t ha[EN / 16][4];
#pragma unroll
    for (int kk = 0; kk < EN / 16; kk++) {
        ha[kk][0] = pack2<T>(acc[2 * kk][0], acc[2 * kk][1]);
        ha[kk][1] = pack2<T>(acc[2 * kk][2], acc[2 * kk][3]);
        ha[kk][2] = pack2<T>(acc[2 * kk + 1][0], acc[2 * kk + 1][1]);
        ha[kk][3] = pack2<T>(acc[2 * kk + 1][2], acc[2 * kk + 1][3]);
    }

    // ---- OUT = base + Hg @ Bcat ----
    for (int sl = 0; sl < nsl; sl++) {
        if (sl + 1 < nsl) {
            load_up(sl + 1, (sl + 1) & 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const unsigned char* bs = smem_apply + (sl & 1) * G::STAGE;
        float o[KS / 8][4];
#pragma unroll
        for (int i = 0; i < KS / 8; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < EN / 16; kk++) {
#pragma unroll
            for (int n2 = 0; n2 < KS / 16; n2++) {
                uint32_t bq[4];
                ldm_x4_t(bq, bs + (kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * G::BP + (n2 * 16 + (lane >> 4) * 8) * 2);
                mma16816<T>(o[2 * n2], ha[kk], bq[0], bq[1]);
                mma16816<T>(o[2 * n2 + 1], ha[kk], bq[2], bq[3]);
            }
        }
        // out = base + o, formed in the base slice (this warp's 16 rows), then stored
        // with 16-byte writes
        unsigned char* os = smem_apply + (sl & 1) * G::STAGE + G::BS;
#pragma unroll
        for (int hr = 0; hr < 2; hr++) {
            unsigned char* orow = os + (16 * warp + g + 8 * hr) * G::OP;
#pragma unroll
            for (int nt = 0; nt < KS / 8; nt++) {
                uint32_t* pp = reinterpret_cast<uint32_t*>(orow + (nt * 8 + 2 * tg) * 2);
                const uint32_t bb = *pp;
                const T* bp = reinterpret_cast<const T*>(&bb);
                *pp = pack2<T>(o[nt][2 * hr] + to_f32(bp[0]), o[nt][2 * hr + 1] + to_f32(bp[1]));
            }
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < (16 * KS / 8) / 32; i++) {
            const int q = lane + 32 * i, row = 16 * warp + q / (KS / 8), pc = q % (KS / 8), tok = t0 + row;
            if (tok < ntok)
                *reinterpret_cast<uint4*>(out + (size_t)tok * C + sl * KS + pc * 8) =
                    *reinterpret_cast<const uint4*>(os + row * G::OP + pc * 16);
        }
        __syncthreads();
    }
}

}  // namespace rwkv

// ===========================================================================
// C ABI
// ===========================================================================
using namespace rwkv;

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

extern "C" size_t rwkv_moe_router_workspace_size(int ntok, int E) {
    if (ntok <= 0 || E <= 0) return 0;
    const size_t nb = (size_t)router_ctas(ntok);
    return align_up(nb * (E + 1) * sizeof(float), 256) + align_up(nb * E * sizeof(int32_t), 256);
}

template <typename T, int EM>
static int launch_router(const void* x, const float* gw, const float* bias, float* logits,
                         int32_t* inds, void* scores, float* pf, int32_t* pc, int ntok, int C,
                         int E, int topk, cudaStream_t st) {
    const int nb = router_ctas(ntok);
    if constexpr (sizeof(T) == 2) {  // tensor-core kernel when its split weights fit
        const size_t smem_mma = (size_t)router_mma_terms<T>() * EM * router_mma_rs(C) * sizeof(T);
        if (smem_mma <= 200 * 1024) {
            auto kern = moe_router_mma_kernel<T, EM / 8>;
            cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_mma);
            if (err != cudaSuccess) return set_cuda_error(err);
            kern<<<nb, ROUTER_WARPS * 32, smem_mma, st>>>((const T*)x, gw, bias, logits, inds, (T*)scores, pf, pc,
                                                          ntok, C, E, topk);
            return check_launch();
        }
    }
    const size_t smem = (size_t)E * C * sizeof(float);
    if (smem > 200 * 1024) return RWKV_ERR_SHAPE;
    auto kern = moe_router_kernel<T, EM>;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return set_cuda_error(err);
    kern<<<nb, ROUTER_WARPS * 32, smem, st>>>((const T*)x, gw, bias, logits, inds, (T*)scores, pf,
                                              pc, ntok, C, E, topk);
    return check_launch();
}

static void launch_finalize(const float* pf, const int32_t* pc, int nb, int ntok, int E, int topk, float* stats,
                            int32_t* counts, cudaStream_t st) {
    if (E <= 8)
        moe_router_finalize_kernel<8><<<1, FIN_THREADS, 0, st>>>(pf, pc, nb, ntok, E, topk, stats, counts);
    else if (E <= 16)
        moe_router_finalize_kernel<16><<<1, FIN_THREADS, 0, st>>>(pf, pc, nb, ntok, E, topk, stats, counts);
    else
        moe_router_finalize_kernel<32><<<1, FIN_THREADS, 0, st>>>(pf, pc, nb, ntok, E, topk, stats, counts);
}

extern "C" int rwkv_moe_router(const void* x, const float* gate_w, const float* bias,
                               float* logits, int32_t* inds, void* scores, float* stats,
                               int32_t* counts, void* workspace, size_t workspace_bytes, int ntok,
                               int C, int E, int topk, int dtype, void* stream) {
    if (ntok <= 0 || C <= 0 || E <= 0 || E > 32 || topk <= 0 || topk > E || topk > 8)
        return RWKV_ERR_SHAPE;
    if (C % 8) return RWKV_ERR_SHAPE;
    if (!x || !gate_w || !inds || !scores || !stats || !workspace) return RWKV_ERR_ARG;
    if (!aligned(x, 16)) return RWKV_ERR_ALIGN;
    if (workspace_bytes < rwkv_moe_router_workspace_size(ntok, E)) return RWKV_ERR_WORKSPACE;
    const int nb = router_ctas(ntok);
    float* pf = (float*)workspace;
    int32_t* pc = (int32_t*)((char*)workspace + align_up((size_t)nb * (E + 1) * sizeof(float), 256));
    cudaStream_t st = (cudaStream_t)stream;
    int rc;
    RWKV_DISPATCH_DTYPE(dtype, T, {
        if (E <= 8)
            rc = launch_router<T, 8>(x, gate_w, bias, logits, inds, scores, pf, pc, ntok, C, E, topk, st);
        else if (E <= 16)
            rc = launch_router<T, 16>(x, gate_w, bias, logits, inds, scores, pf, pc, ntok, C, E, topk, st);
        else
            rc = launch_router<T, 32>(x, gate_w, bias, logits, inds, scores, pf, pc, ntok, C, E, topk, st);
    });
    if (rc) return rc;
    launch_finalize(pf, pc, nb, ntok, E, topk, stats, counts, st);
    return check_launch();
}

extern "C" size_t rwkv_moe_permute_workspace_size(int n_entries, int E) {
    if (n_entries <= 0 || E <= 0) return 0;
    const size_t nb = (size_t)(n_entries + PERM_TILE - 1) / PERM_TILE;
    return 2 * align_up(nb * E * sizeof(int32_t), 256);
}

extern "C" int rwkv_moe_permute(const int32_t* inds, int32_t* perm, int32_t* inv,
                                int32_t* offsets, void* workspace, size_t workspace_bytes,
                                int ntok, int topk, int E, void* stream) {
    if (ntok <= 0 || topk <= 0 || E <= 0 || E > 1024) return RWKV_ERR_SHAPE;
    if ((long long)ntok * topk > 0x7fffffffLL) return RWKV_ERR_SHAPE;
    if (!inds || !perm || !inv || !offsets || !workspace) return RWKV_ERR_ARG;
    const int n = ntok * topk;
    if (workspace_bytes < rwkv_moe_permute_workspace_size(n, E)) return RWKV_ERR_WORKSPACE;
    const int nb = (n + PERM_TILE - 1) / PERM_TILE;
    int32_t* blkcnt = (int32_t*)workspace;
    int32_t* blkoff = (int32_t*)((char*)workspace + align_up((size_t)nb * E * sizeof(int32_t), 256));
    cudaStream_t st = (cudaStream_t)stream;
    moe_count_kernel<<<nb, PERM_THREADS, E * sizeof(int), st>>>(inds, n, E, blkcnt);
    int rc = check_launch();
    if (rc) return rc;
    moe_scan_kernel<<<1, 256, E * sizeof(int), st>>>(blkcnt, nb, E, blkoff, offsets);
    rc = check_launch();
    if (rc) return rc;
    moe_scatter_kernel<<<nb, PERM_THREADS, 2 * (PERM_THREADS / 32) * E * sizeof(int), st>>>(
        inds, n, E, blkoff, perm, inv);
    return check_launch();
}

extern "C" int rwkv_moe_lora_down(const void* x, const void* A, const int32_t* perm,
                                  const int32_t* offsets, float* h, int ntok, int C, int R, int E,
                                  int topk, int dtype, void* stream) {
    if (ntok <= 0 || C <= 0 || E <= 0 || E > 256 || topk <= 0) return RWKV_ERR_SHAPE;
    if (R != 8 && R != 16 && R != 32 && R != 64) return RWKV_ERR_SHAPE;
    if (!x || !A || !perm || !offsets || !h) return RWKV_ERR_ARG;
    const int n = ntok * topk;
    const int grid = (n + 7) / 8 < 148 * 16 ? (n + 7) / 8 : 148 * 16;
    cudaStream_t st = (cudaStream_t)stream;
    RWKV_DISPATCH_DTYPE(dtype, T, {
        switch (R) {
            case 8: moe_lora_down_kernel<T, 8><<<grid, 256, 0, st>>>((const T*)x, (const T*)A, perm, offsets, h, n, C, E, topk); break;
            case 16: moe_lora_down_kernel<T, 16><<<grid, 256, 0, st>>>((const T*)x, (const T*)A, perm, offsets, h, n, C, E, topk); break;
            case 32: moe_lora_down_kernel<T, 32><<<grid, 256, 0, st>>>((const T*)x, (const T*)A, perm, offsets, h, n, C, E, topk); break;
            default: moe_lora_down_kernel<T, 64><<<grid, 256, 0, st>>>((const T*)x, (const T*)A, perm, offsets, h, n, C, E, topk); break;
        }
    });
    return check_launch();
}

extern "C" int rwkv_moe_lora_combine(const void* base, const float* h, const void* B,
                                     const int32_t* inds, const void* scores, const int32_t* inv,
                                     void* out, int ntok, int C, int R, int E, int topk, int dtype,
                                     void* stream) {
    if (ntok <= 0 || C <= 0 || E <= 0 || topk <= 0 || topk > 8) return RWKV_ERR_SHAPE;
    if (R != 8 && R != 16 && R != 32) return RWKV_ERR_SHAPE;
    if (!h || !B || !inds || !scores || !inv || !out) return RWKV_ERR_ARG;
    const int grid = (ntok + 7) / 8 < 148 * 16 ? (ntok + 7) / 8 : 148 * 16;
    cudaStream_t st = (cudaStream_t)stream;
    RWKV_DISPATCH_DTYPE(dtype, T, {
        switch (R) {
            case 8: moe_combine_kernel<T, 8><<<grid, 256, 0, st>>>((const T*)base, h, (const T*)B, inds, (const T*)scores, inv, (T*)out, ntok, C, topk); break;
            case 16: moe_combine_kernel<T, 16><<<grid, 256, 0, st>>>((const T*)base, h, (const T*)B, inds, (const T*)scores, inv, (T*)out, ntok, C, topk); break;
            default: moe_combine_kernel<T, 32><<<grid, 256, 0, st>>>((const T*)base, h, (const T*)B, inds, (const T*)scores, inv, (T*)out, ntok, C, topk); break;
        }
    });
    return check_launch();
}

template <typename T, int EN>
static int launch_apply(const void* x, const void* base, const void* A, const void* B, const int32_t* inds,
                        const void* scores, void* out, int ntok, int C, int R, int E, int topk, cudaStream_t st) {
    auto kern = moe_lora_apply_kernel<T, EN>;
    const int smem = apply::Geo<EN>::SMEM;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return set_cuda_error(err);
    const int grid = (ntok + apply::TM - 1) / apply::TM;
    kern<<<grid, apply::NTH, smem, st>>>((const T*)x, (const T*)base, (const T*)A, (const T*)B, inds, (const T*)scores,
                                         (T*)out, ntok, C, R, E, topk);
    return check_launch();
}
template <typename T>
static int launch_apply_en(const void* x, const void* base, const void* A, const void* B, const int32_t* inds,
                           const void* scores, void* out, int ntok, int C, int R, int E, int topk, cudaStream_t st) {
    switch (E * R) {
        case 32: return launch_apply<T, 32>(x, base, A, B, inds, scores, out, ntok, C, R, E, topk, st);
        case 64: return launch_apply<T, 64>(x, base, A, B, inds, scores, out, ntok, C, R, E, topk, st);
        default: return launch_apply<T, 128>(x, base, A, B, inds, scores, out, ntok, C, R, E, topk, st);
    }
}

namespace rwkv {
template <typename T>
int moe_lora_apply_tc(const void* x, const void* base, const void* A, const void* B, const int32_t* inds,
                      const void* scores, void* out, int ntok, int C, int R, int E, int topk, cudaStream_t st);
int moe_lora_apply_tc_routed(const void* x, const void* base, const void* A, const void* B, const float* gate_w,
                             const float* bias, int32_t* inds, void* scores, void* gsplit, float* part_f,
                             int32_t* part_c, void* out, int ntok, int C, int R, int E, int topk, cudaStream_t st);
int moe_apply_tc_grid(int ntok);
static int g_apply_impl = 0;  // 0 automatic (tcgen05), 1 mma.sync, 2 tcgen05
}  // namespace rwkv

extern "C" int rwkv_moe_set_apply_impl(int impl) {
    if (impl < 0 || impl > 2) return RWKV_ERR_ARG;
    g_apply_impl = impl;
    return RWKV_OK;
}

extern "C" int rwkv_moe_lora_apply_supported(int C, int R, int E, int topk, int dtype) {
    const int en = E * R;
    return (dtype == RWKV_F16 || dtype == RWKV_BF16) && C > 0 && C % 64 == 0 && R > 0 && R % 8 == 0 &&
           (en == 32 || en == 64 || en == 128) && topk > 0 && topk <= 8 && topk <= E;
}

extern "C" int rwkv_moe_lora_apply(const void* x, const void* base, const void* A, const void* B,
                                   const int32_t* inds, const void* scores, void* out, int ntok, int C,
                                   int R, int E, int topk, int dtype, void* stream) {
    if (ntok <= 0) return 0;
    if (dtype != RWKV_F16 && dtype != RWKV_BF16) return RWKV_ERR_DTYPE;
    if (!rwkv_moe_lora_apply_supported(C, R, E, topk, dtype)) return RWKV_ERR_SHAPE;
    if (!x || !A || !B || !inds || !out) return RWKV_ERR_ARG;
    if (!aligned(x, 16) || !aligned(A, 16) || !aligned(B, 16) || !aligned(out, 16) || (base && !aligned(base, 16)))
        return RWKV_ERR_ALIGN;
    cudaStream_t st = (cudaStream_t)stream;
    if (g_apply_impl == 1) {
        if (dtype == RWKV_F16) return launch_apply_en<__half>(x, base, A, B, inds, scores, out, ntok, C, R, E, topk, st);
        return launch_apply_en<__nv_bfloat16>(x, base, A, B, inds, scores, out, ntok, C, R, E, topk, st);
    }
    const int rc = dtype == RWKV_F16
                       ? moe_lora_apply_tc<__half>(x, base, A, B, inds, scores, out, ntok, C, R, E, topk, st)
                       : moe_lora_apply_tc<__nv_bfloat16>(x, base, A, B, inds, scores, out, ntok, C, R, E, topk, st);
    if (rc != APPLY_TC_NO_MAPS) return rc;  // launched (or failed after launching)
    if (g_apply_impl == 2) return RWKV_ERR_CUDA;  // the tcgen05 kernel was asked for explicitly
    clear_error();  // the fallback below succeeds or records its own error
    if (dtype == RWKV_F16) return launch_apply_en<__half>(x, base, A, B, inds, scores, out, ntok, C, R, E, topk, st);
    return launch_apply_en<__nv_bfloat16>(x, base, A, B, inds, scores, out, ntok, C, R, E, topk, st);
}

// ---------------------------------------------------------------------------
// Routed apply: router + adapters in one pass over x (fp16).  Workspace: the split gate
// operand (C / 64 blocks of 4 KB), then the per-CTA routing partials.
static size_t routed_gate_bytes(int C) { return align_up((size_t)(C / 64) * 4096, 256); }

extern "C" int rwkv_moe_lora_apply_routed_supported(int C, int R, int E, int topk, int dtype) {
    return g_apply_impl != 1 && dtype == RWKV_F16 && E <= 16 && rwkv_moe_lora_apply_supported(C, R, E, topk, dtype);
}

extern "C" size_t rwkv_moe_lora_apply_routed_workspace_size(int ntok, int C, int E) {
    if (ntok <= 0 || C <= 0 || E <= 0) return 0;
    const size_t nb = (size_t)moe_apply_tc_grid(ntok);
    return routed_gate_bytes(C) + align_up(nb * (E + 1) * sizeof(float), 256) + align_up(nb * E * sizeof(int32_t), 256);
}

extern "C" int rwkv_moe_lora_apply_routed(const void* x, const void* base, const void* A, const void* B,
                                          const float* gate_w, const float* bias, int32_t* inds, void* scores,
                                          float* stats, int32_t* counts, void* workspace, size_t workspace_bytes,
                                          void* out, int ntok, int C, int R, int E, int topk, int dtype,
                                          void* stream) {
    if (ntok <= 0) return RWKV_ERR_SHAPE;
    if (dtype != RWKV_F16) return RWKV_ERR_DTYPE;
    if (!rwkv_moe_lora_apply_routed_supported(C, R, E, topk, dtype)) return RWKV_ERR_SHAPE;
    if (!x || !A || !B || !gate_w || !inds || !scores || !stats || !out || !workspace) return RWKV_ERR_ARG;
    if (!aligned(x, 16) || !aligned(A, 16) || !aligned(B, 16) || !aligned(out, 16) || (base && !aligned(base, 16)) ||
        !aligned(workspace, 256))
        return RWKV_ERR_ALIGN;
    if (workspace_bytes < rwkv_moe_lora_apply_routed_workspace_size(ntok, C, E)) return RWKV_ERR_WORKSPACE;
    const int nb = moe_apply_tc_grid(ntok);
    unsigned char* ws = (unsigned char*)workspace;
    float* pf = (float*)(ws + routed_gate_bytes(C));
    int32_t* pc = (int32_t*)((unsigned char*)pf + align_up((size_t)nb * (E + 1) * sizeof(float), 256));
    cudaStream_t st = (cudaStream_t)stream;
    const int rc = moe_lora_apply_tc_routed(x, base, A, B, gate_w, bias, inds, scores, ws, pf, pc, out, ntok, C, R,
                                            E, topk, st);
    if (rc == APPLY_TC_NO_MAPS) return RWKV_ERR_CUDA;  // the tensor maps could not be built (message set)
    if (rc) return rc;
    launch_finalize(pf, pc, nb, ntok, E, topk, stats, counts, st);
    return check_launch();
}

extern "C" int rwkv_moe_ortho_loss(const void* A, float* out, int E, int C, int R, int dtype,
                                   void* stream) {
    if (E <= 0 || C <= 0 || R <= 0 || R > 64) return RWKV_ERR_SHAPE;
    if (!A || !out) return RWKV_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    const int threads = R * R < 1024 ? ((R * R + 31) / 32) * 32 : 1024;
    RWKV_DISPATCH_DTYPE(dtype, T, moe_ortho_kernel<T><<<1, threads, 0, st>>>((const T*)A, out, E, C, R));
    return check_launch();
}

// ===========================================================================
// Router entry point that allocates nothing.
//
// Some callers cannot allocate device memory: an FFI binding that only holds the
// device buffers a framework handed it (and has no allocator of its own), or a
// serving loop that reserves all device memory at start-up and must not allocate
// afterwards (cudaMalloc can synchronise the device and fails once the memory is
// reserved).  rwkv_moe_router_noalloc runs the same kernels as rwkv_moe_router,
// with its per-CTA partial sums in the file-scope device array below instead of a
// caller-provided workspace.
// ===========================================================================
#include <cuda.h>

#include <mutex>

namespace rwkv {
constexpr int NOALLOC_MAX_E = 32;
constexpr size_t NOALLOC_SCRATCH_BYTES =
    ((size_t)ROUTER_MAX_CTAS * (NOALLOC_MAX_E + 1) * sizeof(float) + 255) / 256 * 256 +
    ((size_t)ROUTER_MAX_CTAS * NOALLOC_MAX_E * sizeof(int32_t) + 255) / 256 * 256;
// ~75 KB, held by every GPU that loads this library until the process exits.
static __device__ __align__(256) unsigned char g_router_scratch[NOALLOC_SCRATCH_BYTES];

// The address is cached per CUDA context, keyed by the context's unique ID
// (cuCtxGetId): a context that is destroyed and created again (cudaDeviceReset, or the
// primary context released and retained) loads this module again at a new address and
// gets a new ID, so the lookup runs again instead of handing out a stale pointer.
static std::mutex g_scratch_mu;
constexpr int SCRATCH_CACHE = 64;
static unsigned long long g_scratch_ctx[SCRATCH_CACHE];
static void* g_scratch_addr[SCRATCH_CACHE];
static int g_scratch_n = 0;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// ID of the calling thread's current context (0 if it cannot be read: no caching then).
static unsigned long long current_context_id() {
    static CtxGetCurrentFn get_cur = nullptr;
    static CtxGetIdFn get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_cur = reinterpret_cast<CtxGetCurrentFn>(p);
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<CtxGetIdFn>(p);
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!get_cur || !get_id || get_cur(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS) return 0;
    return id;
}

// Device address of g_router_scratch in the current context.  The host-side name is
// only a stand-in, so the address is looked up with the device current, the first
// time the entry point runs in that context (the lookup also makes the runtime bind
// the device's context to the calling thread if it was not yet).
static int router_scratch_address(void** out) {
    unsigned long long id = current_context_id();
    {
        std::lock_guard<std::mutex> lk(g_scratch_mu);
        for (int i = 0; id && i < g_scratch_n; i++)
            if (g_scratch_ctx[i] == id) {
                *out = g_scratch_addr[i];
                return RWKV_OK;
            }
    }
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_router_scratch);
    if (e != cudaSuccess) return set_cuda_error(e);
    id = current_context_id();  // the context is current now
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (id && g_scratch_n < SCRATCH_CACHE) {
        g_scratch_ctx[g_scratch_n] = id;
        g_scratch_addr[g_scratch_n] = p;
        g_scratch_n++;
    }
    *out = p;
    return RWKV_OK;
}
}  // namespace rwkv

extern "C" size_t rwkv_moe_router_noalloc_scratch_bytes(void) { return rwkv::NOALLOC_SCRATCH_BYTES; }

extern "C" int rwkv_moe_router_noalloc(const void* x, const float* gate_w, const float* bias,
                                       float* logits, int32_t* inds, void* scores, float* stats,
                                       int32_t* counts, int ntok, int C, int E, int topk,
                                       int dtype, void* stream) {
    if (ntok <= 0 || C <= 0 || E <= 0 || E > NOALLOC_MAX_E || topk <= 0 || topk > E || topk > 8)
        return RWKV_ERR_SHAPE;
    if (C % 8) return RWKV_ERR_SHAPE;
    if (!x || !gate_w || !inds || !scores || !stats) return RWKV_ERR_ARG;
    if (!aligned(x, 16)) return RWKV_ERR_ALIGN;
    if (rwkv_moe_router_workspace_size(ntok, E) > NOALLOC_SCRATCH_BYTES) return RWKV_ERR_WORKSPACE;
    void* scratch = nullptr;
    int rc = router_scratch_address(&scratch);
    if (rc) return rc;
    const int nb = router_ctas(ntok);
    // every partial is written by its CTA before the finalize kernel reads it, so
    // nothing left in the array by an earlier call needs clearing
    float* pf = (float*)scratch;
    int32_t* pc = (int32_t*)((char*)scratch + align_up((size_t)nb * (E + 1) * sizeof(float), 256));
    cudaStream_t st = (cudaStream_t)stream;
    RWKV_DISPATCH_DTYPE(dtype, T, {
        if (E <= 8)
            rc = launch_router<T, 8>(x, gate_w, bias, logits, inds, scores, pf, pc, ntok, C, E, topk, st);
        else if (E <= 16)
            rc = launch_router<T, 16>(x, gate_w, bias, logits, inds, scores, pf, pc, ntok, C, E, topk, st);
        else
            rc = launch_router<T, 32>(x, gate_w, bias, logits, inds, scores, pf, pc, ntok, C, E, topk, st);
    });
    if (rc) return rc;
    launch_finalize(pf, pc, nb, ntok, E, topk, stats, counts, st);
    return check_launch();
}

static int ep_grid(int n) { return (n + 7) / 8 < 148 * 16 ? (n + 7) / 8 : 148 * 16; }

extern "C" int rwkv_moe_gather_rows(const void* x, const int32_t* perm, void* rows, int n, int C,
                                    int topk, int dtype, void* stream) {
    if (n <= 0 || C <= 0 || topk <= 0) return RWKV_ERR_SHAPE;
    if (!x || !perm || !rows) return RWKV_ERR_ARG;
    if (!aligned(x, 16) || !aligned(rows, 16)) return RWKV_ERR_ALIGN;
    cudaStream_t st = (cudaStream_t)stream;
    RWKV_DISPATCH_DTYPE(dtype, T, {
        if ((C * (int)sizeof(T)) % 16) return RWKV_ERR_SHAPE;
        moe_gather_rows_kernel<T><<<ep_grid(n), 256, 0, st>>>((const T*)x, perm, (T*)rows, n, C, topk);
    });
    return check_launch();
}

extern "C" int rwkv_moe_lora_up(const float* h, const void* B, const int32_t* offsets,
                                const int32_t* out_index, void* y, int n, int C, int R, int E,
                                int dtype, void* stream) {
    if (n <= 0 || C <= 0 || E <= 0 || E > 256) return RWKV_ERR_SHAPE;
    if (R != 8 && R != 16 && R != 32) return RWKV_ERR_SHAPE;
    if (!h || !B || !offsets || !y) return RWKV_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    const int grid = ep_grid(n);
    RWKV_DISPATCH_DTYPE(dtype, T, {
        switch (R) {
            case 8: moe_lora_up_kernel<T, 8><<<grid, 256, 0, st>>>(h, (const T*)B, offsets, out_index, (T*)y, n, C, E); break;
            case 16: moe_lora_up_kernel<T, 16><<<grid, 256, 0, st>>>(h, (const T*)B, offsets, out_index, (T*)y, n, C, E); break;
            default: moe_lora_up_kernel<T, 32><<<grid, 256, 0, st>>>(h, (const T*)B, offsets, out_index, (T*)y, n, C, E); break;
        }
    });
    return check_launch();
}

extern "C" int rwkv_moe_combine_rows(const void* base, const void* rows, const void* scores,
                                     const int32_t* inv, void* out, int ntok, int C, int topk,
                                     int dtype, void* stream) {
    if (ntok <= 0 || C <= 0 || topk <= 0) return RWKV_ERR_SHAPE;
    if (!rows || !scores || !inv || !out) return RWKV_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    RWKV_DISPATCH_DTYPE(dtype, T, {
        const int vec = (C * (int)sizeof(T)) % 16 == 0 && aligned(rows, 16) && aligned(out, 16) &&
                        (!base || aligned(base, 16));
        moe_combine_rows_kernel<T><<<ep_grid(ntok), 256, 0, st>>>((const T*)base, (const T*)rows,
                                                                  (const T*)scores, inv, (T*)out, ntok, C,
                                                                  topk, vec);
    });
    return check_launch();
}

extern "C" int rwkv_moe_expert_mix_rows(const void* x, const void* prev, const void* x_k,
                                        const int32_t* perm, const int32_t* offsets, void* rows,
                                        int n, int Tseq, int C, int topk, int E, int dtype,
                                        void* stream) {
    if (n <= 0 || Tseq <= 0 || C <= 0 || topk <= 0 || E <= 0 || E > 256) return RWKV_ERR_SHAPE;
    if (!x || !x_k || !perm || !offsets || !rows) return RWKV_ERR_ARG;
    if (!aligned(x, 16) || !aligned(x_k, 16) || !aligned(rows, 16) || (prev && !aligned(prev, 16)))
        return RWKV_ERR_ALIGN;
    cudaStream_t st = (cudaStream_t)stream;
    RWKV_DISPATCH_DTYPE(dtype, T, {
        if ((C * (int)sizeof(T)) % 16) return RWKV_ERR_SHAPE;
        moe_expert_mix_rows_kernel<T><<<ep_grid(n), 256, 0, st>>>((const T*)x, (const T*)prev, (const T*)x_k, perm,
                                                                  offsets, (T*)rows, n, Tseq, C, topk, E);
    });
    return check_launch();
}

// WKV-7 recurrence, step-sequential kernels (fp32 state, fp32 arithmetic).
//
//   wkv7_fwd_seq  : forward, one CTA per (b, h, block of 16 value rows); the
//                   rows of a head are independent in the forward (row i only
//                   reads row i of S), so a head is split over 4 CTAs.
//   wkv7_bwd_seq  : exact backward: each chunk of ckpt_len steps is replayed
//                   from its checkpoint in sub-chunks of 8 steps whose states are
//                   kept in shared memory; no division by the decay.
//   wkv7_step     : one RNN step for a batch of sequences (memory bound).
//
// Math (reference rwkv_mlx/kernels/wkv7_metal.py:53-91, model.py:480-483):
//   sa = S a ;  S <- S diag(decay) + sa b^T + v k^T ;  y = S r.
#include "common.cuh"
#include "wkv7.cuh"

namespace rwkv {

// ---------------------------------------------------------------------------
// Forward.  Block = 4 * RPB threads; thread (row, q) owns columns q, q+4, ...,
// q+60 of state row `row` (interleaved so the 4 lanes of a row hit 4 banks).
// ---------------------------------------------------------------------------
template <typename T, typename TW, int RPB, int TCH>
__global__ void __launch_bounds__(RPB * 4)
    wkv7_fwd_seq_kernel(const T* __restrict__ r, const TW* __restrict__ w, const T* __restrict__ k,
                        const T* __restrict__ v, const T* __restrict__ a, const T* __restrict__ b,
                        const float* __restrict__ s0, T* __restrict__ y, float* __restrict__ sT,
                        float* __restrict__ ckpt, float* __restrict__ sa_out, int T_, int H,
                        int ckpt_len) {
    constexpr int N = 64, NT = RPB * 4;
    __shared__ float s_r[TCH][N], s_w[TCH][N], s_k[TCH][N], s_a[TCH][N], s_b[TCH][N];
    __shared__ float s_v[TCH][RPB], s_y[TCH][RPB], s_sa[TCH][RPB];

    const int bh = blockIdx.x, bi = bh / H, hi = bh % H;
    const int row0 = blockIdx.y * RPB;
    const int tid = threadIdx.x, lrow = tid >> 2, q = tid & 3, row = row0 + lrow;
    const size_t tstride = (size_t)H * N;
    const size_t base = ((size_t)bi * T_ * H + hi) * N;  // (bi, t=0, hi, 0)
    const int nck = ckpt ? T_ / ckpt_len : 0;

    float S[16];
    if (s0) {
        const float* p = s0 + ((size_t)bh * N + row) * N;
#pragma unroll
        for (int jj = 0; jj < 16; jj++) S[jj] = p[q + 4 * jj];
    } else {
#pragma unroll
        for (int jj = 0; jj < 16; jj++) S[jj] = 0.f;
    }

    for (int t0 = 0; t0 < T_; t0 += TCH) {
        const int tc = min(TCH, T_ - t0);
        __syncthreads();
        for (int e = tid; e < tc * N; e += NT) {
            const int tt = e / N, j = e % N;
            const size_t off = base + (size_t)(t0 + tt) * tstride + j;
            s_r[tt][j] = ldg_f32(r + off);
            s_w[tt][j] = expf(-expf(ldg_f32(w + off)));
            s_k[tt][j] = ldg_f32(k + off);
            s_a[tt][j] = ldg_f32(a + off);
            s_b[tt][j] = ldg_f32(b + off);
        }
        for (int e = tid; e < tc * RPB; e += NT) {
            const int tt = e / RPB, rr = e % RPB;
            s_v[tt][rr] = ldg_f32(v + base + (size_t)(t0 + tt) * tstride + row0 + rr);
        }
        __syncthreads();
        for (int tt = 0; tt < tc; tt++) {
            float sa = 0.f;
#pragma unroll
            for (int jj = 0; jj < 16; jj++) sa = fmaf(s_a[tt][q + 4 * jj], S[jj], sa);
            sa += __shfl_xor_sync(0xffffffffu, sa, 1);
            sa += __shfl_xor_sync(0xffffffffu, sa, 2);
            const float vv = s_v[tt][lrow];
            float yp = 0.f;
#pragma unroll
            for (int jj = 0; jj < 16; jj++) {
                const int j = q + 4 * jj;
                S[jj] = fmaf(S[jj], s_w[tt][j], fmaf(s_k[tt][j], vv, sa * s_b[tt][j]));
                yp = fmaf(S[jj], s_r[tt][j], yp);
            }
            yp += __shfl_xor_sync(0xffffffffu, yp, 1);
            yp += __shfl_xor_sync(0xffffffffu, yp, 2);
            if (q == 0) {
                s_y[tt][lrow] = yp;
                s_sa[tt][lrow] = sa;
            }
            if (ckpt) {
                const int t = t0 + tt;
                if ((t + 1) % ckpt_len == 0) {
                    float* p = ckpt + (((size_t)bh * nck + t / ckpt_len) * N + row) * N;
#pragma unroll
                    for (int jj = 0; jj < 16; jj++) p[q + 4 * jj] = S[jj];
                }
            }
        }
        __syncthreads();
        for (int e = tid; e < tc * RPB; e += NT) {
            const int tt = e / RPB, rr = e % RPB;
            const size_t off = base + (size_t)(t0 + tt) * tstride + row0 + rr;
            y[off] = from_f32<T>(s_y[tt][rr]);
            if (sa_out) sa_out[off] = s_sa[tt][rr];
        }
    }
    if (sT) {
        float* p = sT + ((size_t)bh * N + row) * N;
#pragma unroll
        for (int jj = 0; jj < 16; jj++) p[q + 4 * jj] = S[jj];
    }
}

// ---------------------------------------------------------------------------
// Exact backward.  One CTA of 64 threads per (b, h).  Thread tid keeps row tid
// of the state gradient G (Grow) and column tid of G (Gcol) in registers, so
// both row sums (dv, du) and column sums (dk, db, dw) are thread-local; the
// forward states of the current 8-step sub-chunk live in shared memory
// (row-major, rows padded to 65 floats: column reads are conflict-free).
// ---------------------------------------------------------------------------
namespace bwdseq {
constexpr int N = 64, SC = 8, LD = 65, NV = 9;
enum { VR = 0, VDEC, VWF, VK, VV, VA, VB, VDY, VU };
constexpr size_t smem_bytes = ((size_t)(SC + 1) * N * LD + (size_t)NV * SC * N + N) * sizeof(float);
}  // namespace bwdseq

template <typename T, typename TW>
__global__ void __launch_bounds__(64, 1)
    wkv7_bwd_seq_kernel(const T* __restrict__ r, const TW* __restrict__ w, const T* __restrict__ k,
                        const T* __restrict__ v, const T* __restrict__ a, const T* __restrict__ b,
                        const T* __restrict__ dy, const float* __restrict__ s0,
                        const float* __restrict__ dsT, const float* __restrict__ ckpt,
                        T* __restrict__ dr, T* __restrict__ dw, T* __restrict__ dk,
                        T* __restrict__ dv, T* __restrict__ da, T* __restrict__ db,
                        float* __restrict__ ds0, int T_, int H, int ckpt_len) {
    using namespace bwdseq;
    extern __shared__ float smem[];
    float* st = smem;                          // [SC+1][N][LD]
    float* vec = st + (SC + 1) * N * LD;       // [NV][SC][N]
    float* du_s = vec + NV * SC * N;           // [N]
#define VEC(kind, s, j) vec[((kind) * SC + (s)) * N + (j)]

    const int tid = threadIdx.x;
    const int bh = blockIdx.x, bi = bh / H, hi = bh % H;
    const size_t tstride = (size_t)H * N;
    const size_t base = ((size_t)bi * T_ * H + hi) * N;
    const int nck = T_ / ckpt_len;

    float Grow[N], Gcol[N];
    if (dsT) {
        const float* p = dsT + (size_t)bh * N * N;
#pragma unroll
        for (int j = 0; j < N; j++) Grow[j] = p[tid * N + j];
#pragma unroll
        for (int i = 0; i < N; i++) Gcol[i] = p[i * N + tid];
    } else {
#pragma unroll
        for (int j = 0; j < N; j++) Grow[j] = 0.f, Gcol[j] = 0.f;
    }

    auto stage = [&](int t_begin, int n) {
        __syncthreads();
        for (int s = 0; s < n; s++) {
            const size_t off = base + (size_t)(t_begin + s) * tstride + tid;
            const float wr = ldg_f32(w + off);
            const float wf = -expf(wr);
            VEC(VR, s, tid) = ldg_f32(r + off);
            VEC(VWF, s, tid) = wf;
            VEC(VDEC, s, tid) = expf(wf);
            VEC(VK, s, tid) = ldg_f32(k + off);
            VEC(VV, s, tid) = ldg_f32(v + off);
            VEC(VA, s, tid) = ldg_f32(a + off);
            VEC(VB, s, tid) = ldg_f32(b + off);
            VEC(VDY, s, tid) = ldg_f32(dy + off);
        }
        __syncthreads();
    };

    const int nchunks = (T_ + ckpt_len - 1) / ckpt_len;
    for (int c = nchunks - 1; c >= 0; c--) {
        const int cs = c * ckpt_len, ce = min(T_, cs + ckpt_len);
        const float* start = (c == 0) ? (s0 ? s0 + (size_t)bh * N * N : nullptr)
                                      : ckpt + ((size_t)bh * nck + (c - 1)) * N * N;
        const int nsub = (ce - cs + SC - 1) / SC;
        for (int p = nsub - 1; p >= 0; p--) {
            const int ps = cs + p * SC, n = min(SC, ce - ps);
            float Srow[N];
            if (start) {
#pragma unroll
                for (int j = 0; j < N; j++) Srow[j] = start[tid * N + j];
            } else {
#pragma unroll
                for (int j = 0; j < N; j++) Srow[j] = 0.f;
            }
            // replay the earlier sub-chunks of this chunk (states not kept)
            for (int pp = 0; pp < p; pp++) {
                stage(cs + pp * SC, SC);
                for (int s = 0; s < SC; s++) {
                    float u = 0.f;
#pragma unroll
                    for (int j = 0; j < N; j++) u = fmaf(VEC(VA, s, j), Srow[j], u);
                    const float vi = VEC(VV, s, tid);
#pragma unroll
                    for (int j = 0; j < N; j++)
                        Srow[j] = fmaf(Srow[j], VEC(VDEC, s, j), fmaf(u, VEC(VB, s, j), vi * VEC(VK, s, j)));
                }
            }
            // replay this sub-chunk keeping every state and sa
            stage(ps, n);
#pragma unroll
            for (int j = 0; j < N; j++) st[tid * LD + j] = Srow[j];
            for (int s = 0; s < n; s++) {
                float u = 0.f;
#pragma unroll
                for (int j = 0; j < N; j++) u = fmaf(VEC(VA, s, j), Srow[j], u);
                const float vi = VEC(VV, s, tid);
#pragma unroll
                for (int j = 0; j < N; j++) {
                    Srow[j] = fmaf(Srow[j], VEC(VDEC, s, j), fmaf(u, VEC(VB, s, j), vi * VEC(VK, s, j)));
                    st[((s + 1) * N + tid) * LD + j] = Srow[j];
                }
                VEC(VU, s, tid) = u;
            }
            __syncthreads();
            // reverse over the sub-chunk
            for (int s = n - 1; s >= 0; s--) {
                const float* Sp = st + (size_t)s * N * LD;
                const float* Sn = st + (size_t)(s + 1) * N * LD;
                const float dyi = VEC(VDY, s, tid), ri = VEC(VR, s, tid);
#pragma unroll
                for (int j = 0; j < N; j++) Grow[j] = fmaf(dyi, VEC(VR, s, j), Grow[j]);
#pragma unroll
                for (int i = 0; i < N; i++) Gcol[i] = fmaf(VEC(VDY, s, i), ri, Gcol[i]);
                float dr_ = 0.f, dv_ = 0.f, du_ = 0.f, dk_ = 0.f, db_ = 0.f, dD = 0.f;
#pragma unroll
                for (int j = 0; j < N; j++) {
                    dv_ = fmaf(Grow[j], VEC(VK, s, j), dv_);
                    du_ = fmaf(Grow[j], VEC(VB, s, j), du_);
                }
#pragma unroll
                for (int i = 0; i < N; i++) {
                    dr_ = fmaf(Sn[i * LD + tid], VEC(VDY, s, i), dr_);
                    dk_ = fmaf(Gcol[i], VEC(VV, s, i), dk_);
                    db_ = fmaf(Gcol[i], VEC(VU, s, i), db_);
                    dD = fmaf(Sp[i * LD + tid], Gcol[i], dD);
                }
                du_s[tid] = du_;
                __syncthreads();
                float da_ = 0.f;
#pragma unroll
                for (int i = 0; i < N; i++) da_ = fmaf(Sp[i * LD + tid], du_s[i], da_);
                const size_t off = base + (size_t)(ps + s) * tstride + tid;
                const float deci = VEC(VDEC, s, tid), ai = VEC(VA, s, tid);
                dr[off] = from_f32<T>(dr_);
                dw[off] = from_f32<T>(dD * deci * VEC(VWF, s, tid));
                dk[off] = from_f32<T>(dk_);
                dv[off] = from_f32<T>(dv_);
                da[off] = from_f32<T>(da_);
                db[off] = from_f32<T>(db_);
#pragma unroll
                for (int j = 0; j < N; j++) Grow[j] = fmaf(Grow[j], VEC(VDEC, s, j), du_ * VEC(VA, s, j));
#pragma unroll
                for (int i = 0; i < N; i++) Gcol[i] = fmaf(Gcol[i], deci, du_s[i] * ai);
                __syncthreads();
            }
        }
    }
    if (ds0) {
        float* p = ds0 + (size_t)bh * N * N + (size_t)tid * N;
#pragma unroll
        for (int j = 0; j < N; j++) p[j] = Grow[j];
    }
#undef VEC
}

// ---------------------------------------------------------------------------
// One RNN step.  One CTA (8 warps) per (sequence, head); warp w owns rows
// 8w..8w+7; lane l owns columns 2l, 2l+1 (one coalesced float2 per row).
// ---------------------------------------------------------------------------
template <typename T, typename TW>
__global__ void __launch_bounds__(256)
    wkv7_step_kernel(float* __restrict__ S, const T* __restrict__ r, const TW* __restrict__ w,
                     const T* __restrict__ k, const T* __restrict__ v, const T* __restrict__ a,
                     const T* __restrict__ b, T* __restrict__ y, int w_mode) {
    constexpr int N = 64;
    __shared__ float sv[N];
    const int bh = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t vbase = (size_t)bh * N;
    if (tid < N) sv[tid] = ldg_f32(v + vbase + tid);
    const int j0 = 2 * lane;
    float2 rj, dj, kj, aj, bj;
    rj.x = ldg_f32(r + vbase + j0), rj.y = ldg_f32(r + vbase + j0 + 1);
    kj.x = ldg_f32(k + vbase + j0), kj.y = ldg_f32(k + vbase + j0 + 1);
    aj.x = ldg_f32(a + vbase + j0), aj.y = ldg_f32(a + vbase + j0 + 1);
    bj.x = ldg_f32(b + vbase + j0), bj.y = ldg_f32(b + vbase + j0 + 1);
    dj.x = ldg_f32(w + vbase + j0), dj.y = ldg_f32(w + vbase + j0 + 1);
    if (w_mode == 0) dj.x = expf(-expf(dj.x)), dj.y = expf(-expf(dj.y));
    __syncthreads();

    float2* Sb = reinterpret_cast<float2*>(S + (size_t)bh * N * N);
    float2 s[8];
    float u[8], yp[8];
#pragma unroll
    for (int rr = 0; rr < 8; rr++) s[rr] = Sb[(warp * 8 + rr) * (N / 2) + lane];
#pragma unroll
    for (int rr = 0; rr < 8; rr++) u[rr] = fmaf(s[rr].x, aj.x, s[rr].y * aj.y);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int rr = 0; rr < 8; rr++) u[rr] += __shfl_xor_sync(0xffffffffu, u[rr], o);
#pragma unroll
    for (int rr = 0; rr < 8; rr++) {
        const float vi = sv[warp * 8 + rr];
        s[rr].x = fmaf(s[rr].x, dj.x, fmaf(u[rr], bj.x, vi * kj.x));
        s[rr].y = fmaf(s[rr].y, dj.y, fmaf(u[rr], bj.y, vi * kj.y));
        Sb[(warp * 8 + rr) * (N / 2) + lane] = s[rr];
        yp[rr] = fmaf(s[rr].x, rj.x, s[rr].y * rj.y);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int rr = 0; rr < 8; rr++) yp[rr] += __shfl_xor_sync(0xffffffffu, yp[rr], o);
    if (lane < 8) {
        float val = yp[0];
#pragma unroll
        for (int rr = 1; rr < 8; rr++)
            if (lane == rr) val = yp[rr];
        y[vbase + warp * 8 + lane] = from_f32<T>(val);
    }
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------
template <typename T, typename TW>
int launch_fwd_seq(const WkvFwdArgs& p, cudaStream_t st) {
    constexpr int RPB = 16, TCH = 32;
    dim3 grid(p.B * p.H, 64 / RPB);
    wkv7_fwd_seq_kernel<T, TW, RPB, TCH><<<grid, RPB * 4, 0, st>>>(
        (const T*)p.r, (const TW*)p.w, (const T*)p.k, (const T*)p.v, (const T*)p.a, (const T*)p.b,
        p.s0, (T*)p.y, p.sT, p.ckpt, p.sa, p.T, p.H, p.ckpt_len);
    return check_launch();
}

template <typename T, typename TW>
int launch_bwd_seq(const WkvBwdArgs& p, cudaStream_t st) {
    auto kern = wkv7_bwd_seq_kernel<T, TW>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)bwdseq::smem_bytes);
    if (e != cudaSuccess) return set_cuda_error(e);
    kern<<<p.B * p.H, 64, bwdseq::smem_bytes, st>>>(
        (const T*)p.r, (const TW*)p.w, (const T*)p.k, (const T*)p.v, (const T*)p.a, (const T*)p.b,
        (const T*)p.dy, p.s0, p.dsT, p.ckpt, (T*)p.dr, (T*)p.dw, (T*)p.dk, (T*)p.dv, (T*)p.da,
        (T*)p.db, p.ds0, p.T, p.H, p.ckpt_len);
    return check_launch();
}

template <typename T, typename TW>
int launch_step(float* S, const void* r, const void* w, const void* k, const void* v,
                const void* a, const void* b, void* y, int Bs, int H, int w_mode, cudaStream_t st) {
    wkv7_step_kernel<T, TW><<<Bs * H, 256, 0, st>>>(S, (const T*)r, (const TW*)w, (const T*)k,
                                                 (const T*)v, (const T*)a, (const T*)b, (T*)y,
                                                 w_mode);
    return check_launch();
}

int wkv7_fwd_seq(const WkvFwdArgs& p, cudaStream_t st) {
    RWKV_DISPATCH_DTYPE_W(p.dtype, p.w_dtype, T, TW, return launch_fwd_seq<T, TW>(p, st));
    return RWKV_OK;
}
int wkv7_bwd_seq(const WkvBwdArgs& p, cudaStream_t st) {
    RWKV_DISPATCH_DTYPE_W(p.dtype, p.w_dtype, T, TW, return launch_bwd_seq<T, TW>(p, st));
    return RWKV_OK;
}
int wkv7_step_launch(float* S, const void* r, const void* w, const void* k, const void* v,
                     const void* a, const void* b, void* y, int Bs, int H, int dtype, int w_dtype,
                     int w_mode, cudaStream_t st) {
    RWKV_DISPATCH_DTYPE_W(dtype, w_dtype, T, TW,
                          return launch_step<T, TW>(S, r, w, k, v, a, b, y, Bs, H, w_mode, st));
    return RWKV_OK;
}

}  // namespace rwkv

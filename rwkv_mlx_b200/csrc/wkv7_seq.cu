// WKV-7 recurrence, step-sequential kernels (fp32 state, fp32 arithmetic).
//
//   wkv7_fwd_seq  : forward, one CTA per (b, h, block of 16 value rows); the
//                   rows of a head are independent in the forward (row i only
//                   reads row i of S), so a head is split over 4 CTAs.
//   wkv7_bwd_seq  : exact backward: each chunk of ckpt_len steps is replayed
//                   from its checkpoint in sub-chunks of 8 steps whose states are
//                   kept in shared memory; no division by the decay.  256 threads
//                   per (b, h), each owning a quarter of a row and of a column of dS.
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
// 256 threads per (b, h): thread (i, q) = (tid / 4, tid % 4) owns the strided quarter
// j = 4 jj + q (jj < 16) of row i of G = dL/dS and of row i of the replayed state, and
// the strided quarter i' = 4 ii + q of column i of G (G is kept twice, by rows and by
// columns, so that row sums (dv, dsa) and column sums (dr, dk, db, dw, da) are both
// thread-local plus a 4-lane shuffle).  Per-step vectors sit in shared memory in the
// same quarter layout ([q][jj]), so a thread reads its 16 elements as 4 float4.
constexpr int N = 64, SC = 8, LDS_ = 72, NT = 256, NVEC = 9, NOUT = 6;
enum { VR = 0, VDEC, VWF, VK, VV, VA, VB, VDY, VU };
constexpr int QS = 20;                            // quarter stride (floats): 4 quarters in distinct banks
constexpr int VROW = 4 * QS;                      // one vector of one step in quarter layout
constexpr int VSZ = SC * VROW;                    // one vector kind for a sub-chunk
constexpr int OSZ = SC * N;                       // one gradient kind for a sub-chunk
constexpr size_t ST_FLOATS = (size_t)(SC + 1) * N * LDS_;
constexpr size_t smem_bytes = (ST_FLOATS + (size_t)NVEC * VSZ + (size_t)NOUT * OSZ + 2 * VROW) * sizeof(float);
__device__ __forceinline__ int qidx(int e) { return (e & 3) * QS + (e >> 2); }  // element e -> [q][jj]
}  // namespace bwdseq

template <typename T, typename TW>
__global__ void __launch_bounds__(bwdseq::NT, 1)
    wkv7_bwd_seq_kernel(const T* __restrict__ r, const TW* __restrict__ w, const T* __restrict__ k,
                        const T* __restrict__ v, const T* __restrict__ a, const T* __restrict__ b,
                        const T* __restrict__ dy, const float* __restrict__ s0,
                        const float* __restrict__ dsT, const float* __restrict__ ckpt,
                        T* __restrict__ dr, T* __restrict__ dw, T* __restrict__ dk,
                        T* __restrict__ dv, T* __restrict__ da, T* __restrict__ db,
                        float* __restrict__ ds0, int T_, int H, int ckpt_len) {
    using namespace bwdseq;
    extern __shared__ __align__(16) float smem[];
    float* st = smem;                 // [SC+1][N][LDS_] replayed states
    float* vec = st + ST_FLOATS;      // [NVEC][SC][4][QS]
    float* outs = vec + NVEC * VSZ;   // [NOUT][SC][N] gradients of the sub-chunk (plain layout)
    float* dus = outs + NOUT * OSZ;   // [2][4][QS] dsa of the current step (double-buffered)

    const int tid = threadIdx.x, i = tid >> 2, q = tid & 3;
    const int bh = blockIdx.x, bi = bh / H, hi = bh % H;
    const size_t tstride = (size_t)H * N;
    const size_t base = ((size_t)bi * T_ * H + hi) * N;
    const int nck = T_ / ckpt_len;
    const int iq = qidx(i);

    auto V4 = [&](int kind, int s, float (&o)[16]) {
        const float4* p = reinterpret_cast<const float4*>(vec + kind * VSZ + s * VROW + q * QS);
#pragma unroll
        for (int m = 0; m < 4; m++) {
            const float4 x = p[m];
            o[4 * m] = x.x, o[4 * m + 1] = x.y, o[4 * m + 2] = x.z, o[4 * m + 3] = x.w;
        }
    };
    auto V1 = [&](int kind, int s) { return vec[kind * VSZ + s * VROW + iq]; };

    float Grow[16], Gcol[16];
    if (dsT) {
        const float* p = dsT + (size_t)bh * N * N;
#pragma unroll
        for (int jj = 0; jj < 16; jj++) Grow[jj] = p[i * N + 4 * jj + q], Gcol[jj] = p[(4 * jj + q) * N + i];
    } else {
#pragma unroll
        for (int jj = 0; jj < 16; jj++) Grow[jj] = 0.f, Gcol[jj] = 0.f;
    }

    auto stage = [&](int t_begin, int n) {
        __syncthreads();
        for (int e = tid; e < SC * N; e += NT) {
            const int s = e / N, j = e % N;
            if (s >= n) continue;
            const size_t off = base + (size_t)(t_begin + s) * tstride + j;
            const float wf = -expf(ldg_f32(w + off));
            const int d = s * VROW + qidx(j);
            vec[VR * VSZ + d] = ldg_f32(r + off);
            vec[VWF * VSZ + d] = wf;
            vec[VDEC * VSZ + d] = expf(wf);
            vec[VK * VSZ + d] = ldg_f32(k + off);
            vec[VV * VSZ + d] = ldg_f32(v + off);
            vec[VA * VSZ + d] = ldg_f32(a + off);
            vec[VB * VSZ + d] = ldg_f32(b + off);
            vec[VDY * VSZ + d] = ldg_f32(dy + off);
        }
        __syncthreads();
    };
    // one forward step of state row i (own quarter); returns sa_i
    auto fwd_step = [&](int s, float (&S)[16]) {
        float av[16], bv[16], kv[16], dc[16];
        V4(VA, s, av), V4(VB, s, bv), V4(VK, s, kv), V4(VDEC, s, dc);
        float u = 0.f;
#pragma unroll
        for (int jj = 0; jj < 16; jj++) u = fmaf(av[jj], S[jj], u);
        u += __shfl_xor_sync(0xffffffffu, u, 1);
        u += __shfl_xor_sync(0xffffffffu, u, 2);
        const float vi = V1(VV, s);
#pragma unroll
        for (int jj = 0; jj < 16; jj++) S[jj] = fmaf(S[jj], dc[jj], fmaf(u, bv[jj], vi * kv[jj]));
        return u;
    };

    int buf = 0;
    const int nchunks = (T_ + ckpt_len - 1) / ckpt_len;
    for (int c = nchunks - 1; c >= 0; c--) {
        const int cs = c * ckpt_len, ce = min(T_, cs + ckpt_len);
        const float* start = (c == 0) ? (s0 ? s0 + (size_t)bh * N * N : nullptr)
                                      : ckpt + ((size_t)bh * nck + (c - 1)) * N * N;
        const int nsub = (ce - cs + SC - 1) / SC;
        for (int p = nsub - 1; p >= 0; p--) {
            const int ps = cs + p * SC, n = min(SC, ce - ps);
            float S[16];
#pragma unroll
            for (int jj = 0; jj < 16; jj++) S[jj] = start ? start[i * N + 4 * jj + q] : 0.f;
            // replay the earlier sub-chunks of this chunk (states not kept)
            for (int pp = 0; pp < p; pp++) {
                stage(cs + pp * SC, SC);
                for (int s = 0; s < SC; s++) fwd_step(s, S);
            }
            // replay this sub-chunk keeping every state and sa
            stage(ps, n);
#pragma unroll
            for (int jj = 0; jj < 16; jj++) st[i * LDS_ + 4 * jj + q] = S[jj];
            for (int s = 0; s < n; s++) {
                const float u = fwd_step(s, S);
                float* dst = st + (size_t)(s + 1) * N * LDS_ + i * LDS_;
#pragma unroll
                for (int jj = 0; jj < 16; jj++) dst[4 * jj + q] = S[jj];
                if (q == 0) vec[VU * VSZ + s * VROW + iq] = u;
            }
            __syncthreads();
            // reverse over the sub-chunk
            for (int s = n - 1; s >= 0; s--) {
                const float* Sp = st + (size_t)s * N * LDS_;
                const float* Sn = st + (size_t)(s + 1) * N * LDS_;
                float rv[16], dyv[16];
                V4(VR, s, rv), V4(VDY, s, dyv);
                const float dyi = V1(VDY, s), ri = V1(VR, s);
#pragma unroll
                for (int jj = 0; jj < 16; jj++) Grow[jj] = fmaf(dyi, rv[jj], Grow[jj]);
#pragma unroll
                for (int ii = 0; ii < 16; ii++) Gcol[ii] = fmaf(dyv[ii], ri, Gcol[ii]);
                float dv_ = 0.f, du_ = 0.f, dr_ = 0.f, dk_ = 0.f, db_ = 0.f, dD = 0.f;
                {
                    float kv[16], bv[16];
                    V4(VK, s, kv), V4(VB, s, bv);
#pragma unroll
                    for (int jj = 0; jj < 16; jj++) dv_ = fmaf(Grow[jj], kv[jj], dv_), du_ = fmaf(Grow[jj], bv[jj], du_);
                }
                {
                    float vv[16], uv[16];
                    V4(VV, s, vv), V4(VU, s, uv);
#pragma unroll
                    for (int ii = 0; ii < 16; ii++) {
                        const int row = 4 * ii + q;
                        dr_ = fmaf(Sn[row * LDS_ + i], dyv[ii], dr_);
                        dk_ = fmaf(Gcol[ii], vv[ii], dk_);
                        db_ = fmaf(Gcol[ii], uv[ii], db_);
                        dD = fmaf(Sp[row * LDS_ + i], Gcol[ii], dD);
                    }
                }
#pragma unroll
                for (int o = 1; o <= 2; o <<= 1) {
                    dv_ += __shfl_xor_sync(0xffffffffu, dv_, o);
                    du_ += __shfl_xor_sync(0xffffffffu, du_, o);
                    dr_ += __shfl_xor_sync(0xffffffffu, dr_, o);
                    dk_ += __shfl_xor_sync(0xffffffffu, dk_, o);
                    db_ += __shfl_xor_sync(0xffffffffu, db_, o);
                    dD += __shfl_xor_sync(0xffffffffu, dD, o);
                }
                float* du_s = dus + buf * VROW;
                if (q == 0) du_s[iq] = du_;
                __syncthreads();
                float duv[16];
                {
                    const float4* pd = reinterpret_cast<const float4*>(du_s + q * QS);
#pragma unroll
                    for (int m = 0; m < 4; m++) {
                        const float4 x = pd[m];
                        duv[4 * m] = x.x, duv[4 * m + 1] = x.y, duv[4 * m + 2] = x.z, duv[4 * m + 3] = x.w;
                    }
                }
                float da_ = 0.f;
#pragma unroll
                for (int ii = 0; ii < 16; ii++) da_ = fmaf(Sp[(4 * ii + q) * LDS_ + i], duv[ii], da_);
                da_ += __shfl_xor_sync(0xffffffffu, da_, 1);
                da_ += __shfl_xor_sync(0xffffffffu, da_, 2);
                const float deci = V1(VDEC, s), ai = V1(VA, s);
                if (q == 0) {
                    outs[0 * OSZ + s * N + i] = dr_;
                    outs[1 * OSZ + s * N + i] = dD * deci * V1(VWF, s);
                } else if (q == 1) {
                    outs[2 * OSZ + s * N + i] = dk_;
                    outs[3 * OSZ + s * N + i] = dv_;
                } else if (q == 2) {
                    outs[4 * OSZ + s * N + i] = da_;
                    outs[5 * OSZ + s * N + i] = db_;
                }
                {
                    float av[16], dc[16];
                    V4(VA, s, av), V4(VDEC, s, dc);
#pragma unroll
                    for (int jj = 0; jj < 16; jj++) Grow[jj] = fmaf(Grow[jj], dc[jj], du_ * av[jj]);
                }
#pragma unroll
                for (int ii = 0; ii < 16; ii++) Gcol[ii] = fmaf(Gcol[ii], deci, duv[ii] * ai);
                buf ^= 1;
            }
            __syncthreads();
            // the sub-chunk's gradients, coalesced
            for (int e = tid; e < NOUT * n * N; e += NT) {
                const int kind = e / (n * N), rem = e % (n * N), s = rem / N, j = rem % N;
                const size_t off = base + (size_t)(ps + s) * tstride + j;
                T* dst = kind == 0 ? dr : kind == 1 ? dw : kind == 2 ? dk : kind == 3 ? dv : kind == 4 ? da : db;
                dst[off] = from_f32<T>(outs[kind * OSZ + s * N + j]);
            }
        }
    }
    if (ds0) {
        float* p = ds0 + (size_t)bh * N * N + (size_t)i * N;
#pragma unroll
        for (int jj = 0; jj < 16; jj++) p[4 * jj + q] = Grow[jj];
    }
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
    // the state rows first: their loads overlap the small per-token loads and the barrier
    float2* Sb = reinterpret_cast<float2*>(S + (size_t)bh * N * N);
    float2 s[8];
#pragma unroll
    for (int rr = 0; rr < 8; rr++) s[rr] = Sb[(warp * 8 + rr) * (N / 2) + lane];
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

    float u[8], yp[8];
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
    kern<<<p.B * p.H, bwdseq::NT, bwdseq::smem_bytes, st>>>(
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

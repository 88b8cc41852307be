// Fused element-wise kernels of the RWKV-v7 block around the WKV-7 and GEMM calls
// (the callers of the hot path, rwkv_mlx/model.py:187-263).  Each replaces a chain
// of separate element-wise passes over (B*T, C) activations with one pass.
//
//   lerp         : out[m] = x + (shift(x) - x) * mix[m]      (model.py:188-196, :260-261)
//   tmix_mid     : decay w, value residual, ICLR a, kk normalisation, k scaling,
//                  WKV's a/b inputs                          (model.py:200-226)
//   tmix_post    : GroupNorm (MLX strided or per-head groups), bonus, gate (model.py:229-239)
//   relu_sq      : relu(x)^2 in place                        (model.py:262)
//   add_layernorm: x += delta; y = LayerNorm(x)              (model.py:315-326)
// Arithmetic is fp32; inputs/outputs in the activation dtype (w in fp32).
#include "common.cuh"

namespace rwkv {

template <typename T>
struct Vec {
    static constexpr int N = 16 / sizeof(T);
    uint4 raw;
    __device__ __forceinline__ void load(const T* p) { raw = *reinterpret_cast<const uint4*>(p); }
    __device__ __forceinline__ void store(T* p) const { *reinterpret_cast<uint4*>(p) = raw; }
    __device__ __forceinline__ float get(int i) const { return to_f32(reinterpret_cast<const T*>(&raw)[i]); }
    __device__ __forceinline__ void set(int i, float v) { reinterpret_cast<T*>(&raw)[i] = from_f32<T>(v); }
    __device__ __forceinline__ void zero() { raw = make_uint4(0, 0, 0, 0); }
};

// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256)
    lerp_kernel(const T* __restrict__ x, const T* prev, const T* __restrict__ mix, T* __restrict__ out,
                T* prev_out, int M, long long rows, int Tlen, int C) {  // prev_out may be prev when Tlen = 1
    constexpr int V = Vec<T>::N;
    const int nv = C / V;
    const long long total = rows * nv;
    for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < total;
         q += (long long)gridDim.x * blockDim.x) {
        const long long row = q / nv;
        const int c0 = (int)(q % nv) * V;
        Vec<T> xv, pv;
        xv.load(x + row * C + c0);
        if (row % Tlen) pv.load(x + (row - 1) * C + c0);
        else if (prev) pv.load(prev + (row / Tlen) * C + c0);  // the token before this sequence
        else pv.zero();
        float xf[V], dx[V];
#pragma unroll
        for (int i = 0; i < V; i++) xf[i] = xv.get(i), dx[i] = pv.get(i) - xf[i];
        for (int m = 0; m < M; m++) {
            Vec<T> mv, ov;
            mv.load(mix + (size_t)m * C + c0);
#pragma unroll
            for (int i = 0; i < V; i++) ov.set(i, fmaf(dx[i], mv.get(i), xf[i]));
            ov.store(out + ((size_t)m * rows + row) * C + c0);
        }
        // the sequence's last token becomes its next shift state (this thread read the
        // same vector of prev above when Tlen = 1)
        if (prev_out && row % Tlen == Tlen - 1) xv.store(prev_out + (row / Tlen) * C + c0);
    }
}

// ---------------------------------------------------------------------------
// Vectorised: each lane owns V consecutive channels (one 16-byte vector); the 64
// channels of a head are 64/V consecutive lanes, reduced with xor shuffles.
template <typename T>
__global__ void __launch_bounds__(256, 4)  // <= 64 registers: 32 warps per SM (125 -> 115 us at config 2)
    tmix_mid_kernel(const T* __restrict__ k, const T* __restrict__ v, const T* __restrict__ wl,
                    const T* __restrict__ al, const T* __restrict__ vl, const T* __restrict__ vfirst,
                    const float* __restrict__ w0, const T* __restrict__ a0, const T* __restrict__ v0,
                    const T* __restrict__ kkp, const T* __restrict__ kap, float* __restrict__ w_out,
                    T* __restrict__ k_out, T* __restrict__ v_out, T* __restrict__ a_out,
                    T* __restrict__ b_out, long long rows, int C, int layer0) {
    constexpr int V = Vec<T>::N, LPH = 64 / V;  // lanes per head
    const long long nvec = rows * (C / V);
    for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q - (threadIdx.x & 31) < nvec;
         q += (long long)gridDim.x * blockDim.x) {
        const bool live = q < nvec;
        const long long row = live ? q / (C / V) : 0;
        const int c0 = live ? (int)(q % (C / V)) * V : 0;
        const size_t o = row * C + c0;
        float kv[V], vv[V], av[V], kk[V], ss = 0.f;
        if (live) {
            Vec<T> K, Vv, WL, AL, A0, KK, KA;
            K.load(k + o), Vv.load(v + o), WL.load(wl + o), AL.load(al + o);
            A0.load(a0 + c0), KK.load(kkp + c0), KA.load(kap + c0);
            float wo[V];
#pragma unroll
            for (int i = 0; i < V; i++) {
                const float s = -(w0[c0 + i] + WL.get(i));
                wo[i] = -(fmaxf(s, 0.f) + __logf(1.f + __expf(-fabsf(s)))) - 0.5f;
                kv[i] = K.get(i);
                vv[i] = Vv.get(i);
                av[i] = 1.f / (1.f + __expf(-(A0.get(i) + AL.get(i))));
                kk[i] = kv[i] * KK.get(i);
                ss = fmaf(kk[i], kk[i], ss);
            }
#pragma unroll
            for (int i = 0; i < V; i += 4)
                *reinterpret_cast<float4*>(w_out + o + i) = make_float4(wo[i], wo[i + 1], wo[i + 2], wo[i + 3]);
            if (!layer0) {
                Vec<T> VL, VF, V0;
                VL.load(vl + o), VF.load(vfirst + o), V0.load(v0 + c0);
#pragma unroll
                for (int i = 0; i < V; i++) {
                    const float gte = 1.f / (1.f + __expf(-(V0.get(i) + VL.get(i))));
                    vv[i] = fmaf(VF.get(i) - vv[i], gte, vv[i]);
                }
            }
            Vec<T> KA2 = KA;
#pragma unroll
            for (int i = 0; i < V; i++) kv[i] = kv[i] * fmaf(av[i] - 1.f, KA2.get(i), 1.f);
        }
#pragma unroll
        for (int off = 1; off < LPH; off <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        if (live) {
            const float inv = 1.f / (sqrtf(ss) + 1e-12f);
            Vec<T> KO, VO, AO, BO;
#pragma unroll
            for (int i = 0; i < V; i++) {
                const float kn = kk[i] * inv;
                KO.set(i, kv[i]), VO.set(i, vv[i]), AO.set(i, -kn), BO.set(i, kn * av[i]);
            }
            KO.store(k_out + o), VO.store(v_out + o), AO.store(a_out + o), BO.store(b_out + o);
        }
    }
}

// ---------------------------------------------------------------------------
// One warp per row.  The row of y is staged in shared memory (fp32, 16-byte stores);
// group statistics: MLX strided groups -- lane g sums its group's C/H members; per-head
// groups -- the lanes holding a head reduce with shuffles (fixed order, deterministic);
// head bonus dots: per-vector partials reduced over the 64/V lanes of a head.
template <typename T>
__global__ void __launch_bounds__(128, 8)  // <= 64 registers: 32 warps per SM
    tmix_post_kernel(const T* __restrict__ y, const T* __restrict__ r, const T* __restrict__ k,
                     const T* __restrict__ v, const T* __restrict__ g, const T* __restrict__ lnw,
                     const T* __restrict__ lnb, const T* __restrict__ rk, T* __restrict__ out,
                     long long rows, int C, int H, float eps, int per_head) {
    constexpr int V = Vec<T>::N, LPH = 64 / V;
    extern __shared__ float sm_post[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* ys = sm_post + (size_t)warp * (((C + 2 * H) + 3) & ~3);  // 16-byte aligned per warp
    float* mean = ys + C;
    float* rstd = mean + H;
    const int gsz = C / H, nv = C / V;
    for (long long row = blockIdx.x * 4LL + warp; row < rows; row += gridDim.x * 4LL) {
        const size_t base = row * C;
        // stage y, bonus dot partials per vector
        // every lane runs NJ vector slots; a head's 64/V lanes are all live or all idle
        // because C is a multiple of 64
        const int NJ = (nv + 31) / 32;  // <= 8 (checked on launch)
        float hd[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            if (j >= NJ) break;
            const int qv = lane + 32 * j;
            float d = 0.f;
            if (qv < nv) {
                Vec<T> Y, R, K, RK;
                Y.load(y + base + qv * V), R.load(r + base + qv * V), K.load(k + base + qv * V), RK.load(rk + qv * V);
#pragma unroll
                for (int i = 0; i < V; i += 4)  // 16-byte stores: a lane's V values are contiguous
                    *reinterpret_cast<float4*>(&ys[qv * V + i]) = make_float4(Y.get(i), Y.get(i + 1), Y.get(i + 2), Y.get(i + 3));
#pragma unroll
                for (int i = 0; i < V; i++) d = fmaf(R.get(i) * K.get(i), RK.get(i), d);
            }
#pragma unroll
            for (int off = 1; off < LPH; off <<= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
            hd[j] = d;
        }
        __syncwarp();
        float hm[8], hr[8];  // per-head grouping: the vector's head statistics, in registers
        if (per_head) {
            // a head's 64 channels are the 64/V vectors of LPH consecutive lanes: sums over
            // the lane's own values, then xor shuffles within those lanes (fixed order)
#pragma unroll
            for (int j = 0; j < 8; j++) {
                if (j >= NJ) break;
                const int qv = lane + 32 * j;
                float s1 = 0.f;
                if (qv < nv) {
#pragma unroll
                    for (int i = 0; i < V; i++) s1 += ys[qv * V + i];
                }
#pragma unroll
                for (int off = 1; off < LPH; off <<= 1) s1 += __shfl_xor_sync(0xffffffffu, s1, off);
                const float mu = s1 * (1.f / 64.f);
                float s2 = 0.f;
                if (qv < nv) {
#pragma unroll
                    for (int i = 0; i < V; i++) { const float dd = ys[qv * V + i] - mu; s2 = fmaf(dd, dd, s2); }
                }
#pragma unroll
                for (int off = 1; off < LPH; off <<= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, off);
                hm[j] = mu;
                hr[j] = rsqrtf(s2 * (1.f / 64.f) + eps);
            }
        } else {
            // MLX strided grouping (channel c in group c % H): one lane per group
            for (int gi = lane; gi < H; gi += 32) {
                // four independent partial sums (gsz = 64 is a multiple of 4): the serial
                // shared-memory chain is a quarter as long
                float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
                for (int m = 0; m < gsz; m += 4) {
                    a0 += ys[gi + H * m], a1 += ys[gi + H * (m + 1)];
                    a2 += ys[gi + H * (m + 2)], a3 += ys[gi + H * (m + 3)];
                }
                const float mu = ((a0 + a1) + (a2 + a3)) / (float)gsz;
                a0 = a1 = a2 = a3 = 0.f;
                for (int m = 0; m < gsz; m += 4) {
                    const float d0 = ys[gi + H * m] - mu, d1 = ys[gi + H * (m + 1)] - mu;
                    const float d2 = ys[gi + H * (m + 2)] - mu, d3 = ys[gi + H * (m + 3)] - mu;
                    a0 = fmaf(d0, d0, a0), a1 = fmaf(d1, d1, a1), a2 = fmaf(d2, d2, a2), a3 = fmaf(d3, d3, a3);
                }
                mean[gi] = mu;
                rstd[gi] = rsqrtf(((a0 + a1) + (a2 + a3)) / (float)gsz + eps);
            }
            __syncwarp();
        }
#pragma unroll
        for (int j = 0; j < 8; j++) {
            if (j >= NJ) break;
            const int qv = lane + 32 * j;
            if (qv >= nv) continue;
            Vec<T> Vv, G, W, Bb, O;
            Vv.load(v + base + qv * V), G.load(g + base + qv * V), W.load(lnw + qv * V), Bb.load(lnb + qv * V);
            float yv[V];
#pragma unroll
            for (int i = 0; i < V; i += 4) {
                const float4 q4 = *reinterpret_cast<const float4*>(&ys[qv * V + i]);
                yv[i] = q4.x, yv[i + 1] = q4.y, yv[i + 2] = q4.z, yv[i + 3] = q4.w;
            }
            if (per_head) {
#pragma unroll
                for (int i = 0; i < V; i++) {
                    float o = fmaf((yv[i] - hm[j]) * hr[j], W.get(i), Bb.get(i));
                    o = fmaf(hd[j], Vv.get(i), o);
                    O.set(i, o * G.get(i));
                }
            } else {
                // group of channel c = c % H: one modulo per vector, then increments
                int gi = (qv * V) % H;
#pragma unroll
                for (int i = 0; i < V; i++) {
                    float o = fmaf((yv[i] - mean[gi]) * rstd[gi], W.get(i), Bb.get(i));
                    o = fmaf(hd[j], Vv.get(i), o);
                    O.set(i, o * G.get(i));
                    if (++gi == H) gi = 0;
                }
            }
            O.store(out + base + qv * V);
        }
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------
// The activations between the two stages of the stacked TimeMix LoRA products, h (4, n):
// tanh on slice 1 (decay), sigmoid on slice 3 (gate), slices 0 and 2 untouched
// (model.py:204, :212).  One launch instead of two.
template <typename T>
__global__ void __launch_bounds__(256) lora_act_kernel(T* __restrict__ h, long long nvec) {
    constexpr int V = Vec<T>::N;
    for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < 2 * nvec;
         q += (long long)gridDim.x * blockDim.x) {
        const bool gate = q >= nvec;
        T* p = h + ((gate ? 3 : 1) * nvec + (gate ? q - nvec : q)) * V;
        Vec<T> a;
        a.load(p);
#pragma unroll
        for (int i = 0; i < V; i++) {
            const float f = a.get(i);
            a.set(i, gate ? 1.f / (1.f + expf(-f)) : tanhf(f));
        }
        a.store(p);
    }
}

template <typename T>
__global__ void __launch_bounds__(256) relu_sq_kernel(T* __restrict__ x, long long nvec) {
    constexpr int V = Vec<T>::N;
    for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < nvec;
         q += (long long)gridDim.x * blockDim.x) {
        Vec<T> a;
        a.load(x + q * V);
#pragma unroll
        for (int i = 0; i < V; i++) {
            const float f = fmaxf(a.get(i), 0.f);
            a.set(i, f * f);
        }
        a.store(x + q * V);
    }
}

// ---------------------------------------------------------------------------
// one warp per row: x_out = x (+ delta); y = (x_out - mean) / sqrt(var + eps) * w + b
template <typename T>
__global__ void __launch_bounds__(256)
    add_layernorm_kernel(const T* x, const T* __restrict__ delta, const T* __restrict__ w,
                         const T* __restrict__ b, T* x_out, T* __restrict__ y, long long rows, int C,
                         float eps) {
    constexpr int V = Vec<T>::N;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nv = C / V;
    for (long long row = blockIdx.x * 8LL + warp; row < rows; row += gridDim.x * 8LL) {
        const size_t base = row * C;
        float s = 0.f;
        for (int q = lane; q < nv; q += 32) {
            Vec<T> a;
            a.load(x + base + q * V);
            if (delta) {
                Vec<T> d;
                d.load(delta + base + q * V);
#pragma unroll
                for (int i = 0; i < V; i++) a.set(i, a.get(i) + d.get(i));
                a.store(x_out + base + q * V);
            }
#pragma unroll
            for (int i = 0; i < V; i++) s += a.get(i);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        const float mean = s / (float)C;
        const T* src = delta ? x_out : x;
        __syncwarp();
        float s2 = 0.f;
        for (int q = lane; q < nv; q += 32) {
            Vec<T> a;
            a.load(src + base + q * V);
#pragma unroll
            for (int i = 0; i < V; i++) {
                const float d = a.get(i) - mean;
                s2 = fmaf(d, d, s2);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
        const float rs = rsqrtf(s2 / (float)C + eps);
        for (int q = lane; q < nv; q += 32) {
            Vec<T> a, wv, bv, o;
            a.load(src + base + q * V);
            wv.load(w + q * V);
            bv.load(b + q * V);
#pragma unroll
            for (int i = 0; i < V; i++) o.set(i, fmaf((a.get(i) - mean) * rs, wv.get(i), bv.get(i)));
            o.store(y + base + q * V);
        }
    }
}

// ---------------------------------------------------------------------------
// Greedy decoding's argmax over each row of the logits (first index of the maximum, as
// torch.argmax), written as int64 token ids: one CTA per row, 16-byte vectors.
template <typename T>
__global__ void __launch_bounds__(256)
    argmax_rows_kernel(const T* __restrict__ x, long long ld, long long rows, int V, int64_t* __restrict__ out) {
    constexpr int NV = Vec<T>::N;
    __shared__ float sv[8];
    __shared__ int si[8];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool vec = ((reinterpret_cast<uintptr_t>(x) | (uintptr_t)(ld * sizeof(T))) % 16 == 0) && V % NV == 0;
    for (long long row = blockIdx.x; row < rows; row += gridDim.x) {
        const T* p = x + row * ld;
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        if (vec) {
            for (int j = tid * NV; j < V; j += 256 * NV) {
                Vec<T> a;
                a.load(p + j);
#pragma unroll
                for (int i = 0; i < NV; i++) {
                    const float f = a.get(i);
                    if (f > bv) bv = f, bi = j + i;  // ascending within the thread: first index kept
                }
            }
        } else {
            for (int j = tid; j < V; j += 256) {
                const float f = to_f32(p[j]);
                if (f > bv) bv = f, bi = j;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) bv = ov, bi = oi;
        }
        if (lane == 0) sv[warp] = bv, si[warp] = bi;
        __syncthreads();
        if (tid == 0) {
            for (int w = 1; w < 8; w++)
                if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) bv = sv[w], bi = si[w];
            out[row] = bi == 0x7fffffff ? 0 : bi;
        }
        __syncthreads();
    }
}

// add_layernorm with the row held in registers (NVL 16-byte vectors per lane, C <= 256 V):
// one read of x / delta instead of three passes, the same summation order and roundings
// as add_layernorm_kernel (identical results); in decode every pass was a memory round trip.
template <typename T, int NVL>
__global__ void __launch_bounds__(256)
    add_layernorm_reg_kernel(const T* x, const T* __restrict__ delta, const T* __restrict__ w,
                             const T* __restrict__ b, T* x_out, T* __restrict__ y, long long rows, int C,
                             float eps) {
    constexpr int V = Vec<T>::N;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nv = C / V;
    for (long long row = blockIdx.x * 8LL + warp; row < rows; row += gridDim.x * 8LL) {
        const size_t base = row * C;
        float a[NVL][V];
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < NVL; j++) {
            const int q = lane + 32 * j;
            if (q < nv) {
                Vec<T> xv;
                xv.load(x + base + q * V);
                if (delta) {
                    Vec<T> d;
                    d.load(delta + base + q * V);
#pragma unroll
                    for (int i = 0; i < V; i++) xv.set(i, xv.get(i) + d.get(i));
                    xv.store(x_out + base + q * V);
                }
#pragma unroll
                for (int i = 0; i < V; i++) a[j][i] = xv.get(i), s += a[j][i];
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        const float mean = s / (float)C;
        float s2 = 0.f;
#pragma unroll
        for (int j = 0; j < NVL; j++)
            if (lane + 32 * j < nv) {
#pragma unroll
                for (int i = 0; i < V; i++) {
                    const float d = a[j][i] - mean;
                    s2 = fmaf(d, d, s2);
                }
            }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
        const float rs = rsqrtf(s2 / (float)C + eps);
#pragma unroll
        for (int j = 0; j < NVL; j++) {
            const int q = lane + 32 * j;
            if (q < nv) {
                Vec<T> wv, bv, o;
                wv.load(w + q * V);
                bv.load(b + q * V);
#pragma unroll
                for (int i = 0; i < V; i++) o.set(i, fmaf((a[j][i] - mean) * rs, wv.get(i), bv.get(i)));
                o.store(y + base + q * V);
            }
        }
    }
}

static int grid_for(long long work, int per_block) {
    long long g = (work + per_block - 1) / per_block;
    return (int)(g < 148 * 32 ? (g > 0 ? g : 1) : 148 * 32);
}

}  // namespace rwkv

using namespace rwkv;

static int lerp_launch(const void* x, const void* prev, const void* mix, void* out, void* prev_out, int M,
                       long long rows, int T, int C, int dtype, void* stream) {
    if (M <= 0 || rows <= 0 || T <= 0 || C <= 0 || rows % T) return RWKV_ERR_SHAPE;
    if (!x || !mix || !out) return RWKV_ERR_ARG;
    if (prev_out && prev_out == prev && T != 1) return RWKV_ERR_ARG;  // other threads read prev
    if (!aligned(x, 16) || !aligned(mix, 16) || !aligned(out, 16) || (prev && !aligned(prev, 16)) ||
        (prev_out && !aligned(prev_out, 16)))
        return RWKV_ERR_ALIGN;
    cudaStream_t st = (cudaStream_t)stream;
    RWKV_DISPATCH_DTYPE(dtype, T_, {
        if (C % Vec<T_>::N) return RWKV_ERR_SHAPE;
        lerp_kernel<T_><<<grid_for(rows * (C / Vec<T_>::N), 256), 256, 0, st>>>(
            (const T_*)x, (const T_*)prev, (const T_*)mix, (T_*)out, (T_*)prev_out, M, rows, T, C);
    });
    return check_launch();
}

extern "C" int rwkv_lerp_prev(const void* x, const void* prev, const void* mix, void* out, int M,
                              long long rows, int T, int C, int dtype, void* stream) {
    return lerp_launch(x, prev, mix, out, nullptr, M, rows, T, C, dtype, stream);
}

extern "C" int rwkv_lerp_prev_state(const void* x, const void* prev, const void* mix, void* out, void* prev_out,
                                    int M, long long rows, int T, int C, int dtype, void* stream) {
    return lerp_launch(x, prev, mix, out, prev_out, M, rows, T, C, dtype, stream);
}

extern "C" int rwkv_lerp(const void* x, const void* mix, void* out, int M, long long rows, int T,
                         int C, int dtype, void* stream) {
    return rwkv_lerp_prev(x, nullptr, mix, out, M, rows, T, C, dtype, stream);
}

extern "C" int rwkv_tmix_mid(const void* k, const void* v, const void* wl, const void* al,
                             const void* vl, const void* v_first, const float* w0, const void* a0,
                             const void* v0, const void* k_k, const void* k_a, float* w_out,
                             void* k_out, void* v_out, void* a_out, void* b_out, long long rows,
                             int C, int layer0, int dtype, void* stream) {
    if (rows <= 0 || C <= 0 || C % 64) return RWKV_ERR_SHAPE;
    {
        const void* ps[16] = {k, v, wl, al, vl, v_first, w0, a0, v0, k_k, k_a, w_out, k_out, v_out, a_out, b_out};
        for (const void* p : ps)
            if (p && !aligned(p, 16)) return RWKV_ERR_ALIGN;
    }
    if (!k || !v || !wl || !al || !w0 || !a0 || !k_k || !k_a || !w_out || !k_out || !v_out || !a_out || !b_out)
        return RWKV_ERR_ARG;
    if (!layer0 && (!vl || !v_first || !v0)) return RWKV_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    RWKV_DISPATCH_DTYPE(dtype, T_, tmix_mid_kernel<T_><<<grid_for(rows * (C / Vec<T_>::N), 256), 256, 0, st>>>(
                                       (const T_*)k, (const T_*)v, (const T_*)wl, (const T_*)al, (const T_*)vl,
                                       (const T_*)v_first, w0, (const T_*)a0, (const T_*)v0, (const T_*)k_k,
                                       (const T_*)k_a, w_out, (T_*)k_out, (T_*)v_out, (T_*)a_out, (T_*)b_out,
                                       rows, C, layer0));
    return check_launch();
}

extern "C" int rwkv_tmix_post(const void* y, const void* r, const void* k, const void* v,
                              const void* g, const void* ln_w, const void* ln_b, const void* r_k,
                              void* out, long long rows, int C, int H, float eps, int per_head,
                              int dtype, void* stream) {
    if (rows <= 0 || C <= 0 || H <= 0 || C % H || C / H != 64) return RWKV_ERR_SHAPE;
    if (!y || !r || !k || !v || !g || !ln_w || !ln_b || !r_k || !out) return RWKV_ERR_ARG;
    {
        const void* ps[9] = {y, r, k, v, g, ln_w, ln_b, r_k, out};
        for (const void* p : ps)
            if (!aligned(p, 16)) return RWKV_ERR_ALIGN;
    }
    cudaStream_t st = (cudaStream_t)stream;
    const size_t smem = 4 * (size_t)(((C + 2 * H) + 3) & ~3) * sizeof(float);
    {
        const int V = dtype == RWKV_F32 ? 4 : 8;
        if (C / V > 8 * 32) return RWKV_ERR_SHAPE;  // <= 8 vectors per lane
    }
    RWKV_DISPATCH_DTYPE(dtype, T_, tmix_post_kernel<T_><<<grid_for(rows, 4), 128, smem, st>>>(
                                       (const T_*)y, (const T_*)r, (const T_*)k, (const T_*)v, (const T_*)g,
                                       (const T_*)ln_w, (const T_*)ln_b, (const T_*)r_k, (T_*)out, rows, C, H, eps,
                                       per_head));
    return check_launch();
}

extern "C" int rwkv_relu_sq(void* x, long long n, int dtype, void* stream) {
    if (n <= 0) return RWKV_ERR_SHAPE;
    if (!x) return RWKV_ERR_ARG;
    if (!aligned(x, 16)) return RWKV_ERR_ALIGN;
    cudaStream_t st = (cudaStream_t)stream;
    RWKV_DISPATCH_DTYPE(dtype, T_, {
        if (n % Vec<T_>::N) return RWKV_ERR_SHAPE;
        relu_sq_kernel<T_><<<grid_for(n / Vec<T_>::N, 256), 256, 0, st>>>((T_*)x, n / Vec<T_>::N);
    });
    return check_launch();
}

extern "C" int rwkv_lora_act(void* h, long long n, int dtype, void* stream) {
    if (n <= 0) return RWKV_ERR_SHAPE;
    if (!h) return RWKV_ERR_ARG;
    if (!aligned(h, 16)) return RWKV_ERR_ALIGN;
    cudaStream_t st = (cudaStream_t)stream;
    RWKV_DISPATCH_DTYPE(dtype, T_, {
        if (n % Vec<T_>::N) return RWKV_ERR_SHAPE;
        lora_act_kernel<T_><<<grid_for(2 * (n / Vec<T_>::N), 256), 256, 0, st>>>((T_*)h, n / Vec<T_>::N);
    });
    return check_launch();
}

extern "C" int rwkv_add_layernorm(const void* x, const void* delta, const void* w, const void* b,
                                  void* x_out, void* y, long long rows, int C, float eps, int dtype,
                                  void* stream) {
    if (rows <= 0 || C <= 0) return RWKV_ERR_SHAPE;
    if (!x || !w || !b || !y || (delta && !x_out)) return RWKV_ERR_ARG;
    const void* ps[6] = {x, delta, w, b, x_out, y};
    for (const void* p : ps)
        if (p && !aligned(p, 16)) return RWKV_ERR_ALIGN;
    cudaStream_t st = (cudaStream_t)stream;
    RWKV_DISPATCH_DTYPE(dtype, T_, {
        if (C % Vec<T_>::N) return RWKV_ERR_SHAPE;
        const int nvl = (C / Vec<T_>::N + 31) / 32;
        auto reg = [&](auto kern) {
            kern<<<grid_for(rows, 8), 256, 0, st>>>((const T_*)x, (const T_*)delta, (const T_*)w, (const T_*)b,
                                                    (T_*)x_out, (T_*)y, rows, C, eps);
        };
        if (nvl <= 1) reg(add_layernorm_reg_kernel<T_, 1>);
        else if (nvl <= 2) reg(add_layernorm_reg_kernel<T_, 2>);
        else if (nvl <= 3) reg(add_layernorm_reg_kernel<T_, 3>);
        else if (nvl <= 4) reg(add_layernorm_reg_kernel<T_, 4>);
        else if (nvl <= 8) reg(add_layernorm_reg_kernel<T_, 8>);
        else
            add_layernorm_kernel<T_><<<grid_for(rows, 8), 256, 0, st>>>(
                (const T_*)x, (const T_*)delta, (const T_*)w, (const T_*)b, (T_*)x_out, (T_*)y, rows, C, eps);
    });
    return check_launch();
}

extern "C" int rwkv_argmax_rows(const void* x, long long ld, long long rows, int V, int64_t* out, int dtype,
                                void* stream) {
    if (rows <= 0 || V <= 0 || ld < V) return RWKV_ERR_SHAPE;
    if (!x || !out) return RWKV_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    const int grid = rows < 148 * 16 ? (int)rows : 148 * 16;
    RWKV_DISPATCH_DTYPE(dtype, T_, argmax_rows_kernel<T_><<<grid, 256, 0, st>>>((const T_*)x, ld, rows, V, out));
    return check_launch();
}

// Cross-entropy with the L2 max-logit term of rwkv_mlx/train.py:317-362, evaluated over
// vocabulary chunks so that the full (tokens x vocab) logits never exist at once:
//   ce_chunk       one pass over a chunk of logit columns per token: online softmax
//                  statistics (running max m, running sum s of exp(l - m)), the first
//                  index of the maximum, and the target's logit when the target column
//                  falls in the chunk;
//   ce_finalize    loss = sum_i w_i (log s_i + m_i - l_i,target) / den
//                       + l2_factor * 0.5 * sum_i m_i^2,
//                  w_i = mask_i (den = sum w + 1e-9) or 1 (den = ntok);
//   ce_chunk_grad  d loss / d logits for a chunk, scaled by the incoming gradient g:
//                  g * w_i / den * (softmax_ij - [j = target_i]) + g * l2_factor * m_i * [j = argmax_i],
//                  or (scaled = 0) the same times den / g, whose entries stay O(1) in 16-bit
//                  types; the caller applies g / den to the products it forms from them.
// The per-token state is float4 {m, s, target logit, argmax (int bits)}.
#include "common.cuh"

namespace rwkv {
namespace {

constexpr int WARPS = 8;

__device__ __forceinline__ void merge(float& m, float& s, int& am, float m2, float s2, int am2) {
    // combine two (max, sum exp(. - max), first argmax) partial states; ties keep the
    // lower column index
    if (m2 > m || (m2 == m && am2 < am)) {
        if (m2 > m) {
            s = s * __expf(m - m2) + s2;
            m = m2;
        } else {
            s += s2;
        }
        am = am2;
    } else {
        s += s2 * __expf(m2 - m);
    }
}

template <typename T>
__global__ void __launch_bounds__(WARPS * 32)
    ce_chunk_kernel(const T* __restrict__ logits, long long ld, const int32_t* __restrict__ targets,
                    float4* __restrict__ state, int ntok, int col0, int ncols, int first) {
    constexpr int V = 16 / sizeof(T);
    const bool vec = ((reinterpret_cast<uintptr_t>(logits) | (uintptr_t)(ld * sizeof(T))) % 16 == 0) && ncols % V == 0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = blockIdx.x * WARPS + warp; i < ntok; i += gridDim.x * WARPS) {
        const T* row = logits + (size_t)i * ld;
        float m = -INFINITY, s = 0.f;
        int am = 0x7fffffff;
        if (vec) {  // one 16-byte vector of V columns per lane step
            for (int j = lane * V; j < ncols; j += 32 * V) {
                const uint4 raw = *reinterpret_cast<const uint4*>(row + j);
                const T* e = reinterpret_cast<const T*>(&raw);
                float l[V], lm = -INFINITY;
                int li = 0;
#pragma unroll
                for (int q = 0; q < V; q++) {
                    l[q] = to_f32(e[q]);
                    if (l[q] > lm) lm = l[q], li = q;
                }
                if (lm > m) {
                    s *= __expf(m - lm);
                    m = lm;
                    am = col0 + j + li;
                }
#pragma unroll
                for (int q = 0; q < V; q++) s += __expf(l[q] - m);
            }
        } else {
            for (int j = lane; j < ncols; j += 32) {
                const float l = to_f32(row[j]);
                if (l > m) {
                    s = s * __expf(m - l) + 1.f;
                    m = l;
                    am = col0 + j;
                } else {
                    s += __expf(l - m);
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
            const int am2 = __shfl_xor_sync(0xffffffffu, am, o);
            if (s2 > 0.f) {
                if (s > 0.f)
                    merge(m, s, am, m2, s2, am2);
                else
                    m = m2, s = s2, am = am2;
            }
        }
        if (lane == 0) {
            const int tg = targets[i] - col0;
            float4 st = first ? make_float4(-INFINITY, 0.f, 0.f, __int_as_float(0x7fffffff)) : state[i];
            if (tg >= 0 && tg < ncols) st.z = to_f32(row[tg]);
            float M = st.x, S = st.y;
            int AM = __float_as_int(st.w);
            if (S > 0.f)
                merge(M, S, AM, m, s, am);
            else
                M = m, S = s, AM = am;
            st.x = M, st.y = S, st.w = __int_as_float(AM);
            state[i] = st;
        }
    }
}

// One block; fixed-order reduction (deterministic).
__global__ void __launch_bounds__(1024)
    ce_finalize_kernel(const float4* __restrict__ state, const float* __restrict__ mask, float l2_factor,
                       float* __restrict__ out, int ntok) {
    __shared__ double red[3][32];
    double ce = 0.0, wsum = 0.0, l2 = 0.0;
    for (int i = threadIdx.x; i < ntok; i += blockDim.x) {
        const float4 st = state[i];
        const double w = mask ? (double)mask[i] : 1.0;
        ce += w * ((double)logf(st.y) + (double)st.x - (double)st.z);
        wsum += w;
        l2 += (double)st.x * (double)st.x;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ce += __shfl_xor_sync(0xffffffffu, ce, o);
        wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
        l2 += __shfl_xor_sync(0xffffffffu, l2, o);
    }
    if (lane == 0) red[0][warp] = ce, red[1][warp] = wsum, red[2][warp] = l2;
    __syncthreads();
    if (threadIdx.x == 0) {
        double c = 0.0, w = 0.0, q = 0.0;
        for (int k = 0; k < (int)(blockDim.x >> 5); k++) c += red[0][k], w += red[1][k], q += red[2][k];
        const double den = mask ? w + 1e-9 : (double)ntok;
        const double cterm = c / den, l2term = (double)l2_factor * 0.5 * q;
        out[0] = (float)(cterm + l2term);
        out[1] = (float)cterm;
        out[2] = (float)l2term;
        out[3] = (float)den;
    }
}

template <typename T>
__global__ void __launch_bounds__(WARPS * 32)
    ce_chunk_grad_kernel(const T* logits, long long ld, const int32_t* __restrict__ targets,
                         const float4* __restrict__ state, const float* __restrict__ mask,
                         const float* __restrict__ out, const float* __restrict__ g, float l2_factor, int scaled,
                         T* dlogits, long long ld_out, int ntok, int col0, int ncols) {  // may alias logits
    constexpr int V = 16 / sizeof(T);
    const bool vec = ((reinterpret_cast<uintptr_t>(logits) | reinterpret_cast<uintptr_t>(dlogits) |
                       (uintptr_t)(ld * sizeof(T)) | (uintptr_t)(ld_out * sizeof(T))) % 16 == 0) &&
                     ncols % V == 0;
    const float gv = *g, den = out[3];
    const float c1 = scaled ? gv / den : 1.f, c2 = scaled ? gv * l2_factor : l2_factor * den;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = blockIdx.x * WARPS + warp; i < ntok; i += gridDim.x * WARPS) {
        const float4 st = state[i];
        const float lse = st.x + logf(st.y);
        const float a = c1 * (mask ? mask[i] : 1.f);
        const int tg = targets[i] - col0, am = __float_as_int(st.w) - col0;
        const float l2g = c2 * st.x;
        const T* row = logits + (size_t)i * ld;
        T* drow = dlogits + (size_t)i * ld_out;
        if (vec) {
            for (int j = lane * V; j < ncols; j += 32 * V) {
                const uint4 raw = *reinterpret_cast<const uint4*>(row + j);
                const T* e = reinterpret_cast<const T*>(&raw);
                uint4 o;
                T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
                for (int q = 0; q < V; q++) {
                    float d = a * (__expf(to_f32(e[q]) - lse) - (j + q == tg ? 1.f : 0.f));
                    if (j + q == am) d += l2g;
                    oe[q] = from_f32<T>(d);
                }
                *reinterpret_cast<uint4*>(drow + j) = o;
            }
        } else {
            for (int j = lane; j < ncols; j += 32) {
                float d = a * (__expf(to_f32(row[j]) - lse) - (j == tg ? 1.f : 0.f));
                if (j == am) d += l2g;
                drow[j] = from_f32<T>(d);
            }
        }
    }
}

int ce_grid(int ntok) {
    const int b = (ntok + WARPS - 1) / WARPS;
    return b < 148 * 16 ? b : 148 * 16;
}

}  // namespace
}  // namespace rwkv

using namespace rwkv;

extern "C" int rwkv_ce_chunk(const void* logits, long long ld, const int32_t* targets, float* state,
                             int ntok, int col0, int ncols, int first, int dtype, void* stream) {
    if (ntok <= 0 || ncols <= 0 || col0 < 0 || ld < ncols) return RWKV_ERR_SHAPE;
    if (!logits || !targets || !state) return RWKV_ERR_ARG;
    if (!aligned(state, 16)) return RWKV_ERR_ALIGN;
    cudaStream_t st = (cudaStream_t)stream;
    RWKV_DISPATCH_DTYPE(dtype, T, ce_chunk_kernel<T><<<ce_grid(ntok), WARPS * 32, 0, st>>>(
                                      (const T*)logits, ld, targets, (float4*)state, ntok, col0, ncols, first));
    return check_launch();
}

extern "C" int rwkv_ce_finalize(const float* state, const float* mask, float l2_factor, float* out, int ntok,
                                void* stream) {
    if (ntok <= 0) return RWKV_ERR_SHAPE;
    if (!state || !out) return RWKV_ERR_ARG;
    if (!aligned(state, 16)) return RWKV_ERR_ALIGN;
    ce_finalize_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>((const float4*)state, mask, l2_factor, out, ntok);
    return check_launch();
}

extern "C" int rwkv_ce_chunk_grad(const void* logits, long long ld, const int32_t* targets, const float* state,
                                  const float* mask, const float* out, const float* g, float l2_factor,
                                  int scaled, void* dlogits, long long ld_out, int ntok, int col0, int ncols,
                                  int dtype, void* stream) {
    if (ntok <= 0 || ncols <= 0 || col0 < 0 || ld < ncols || ld_out < ncols) return RWKV_ERR_SHAPE;
    if (!logits || !targets || !state || !out || !g || !dlogits) return RWKV_ERR_ARG;
    if (!aligned(state, 16)) return RWKV_ERR_ALIGN;
    cudaStream_t st = (cudaStream_t)stream;
    RWKV_DISPATCH_DTYPE(dtype, T, ce_chunk_grad_kernel<T><<<ce_grid(ntok), WARPS * 32, 0, st>>>(
                                      (const T*)logits, ld, targets, (const float4*)state, mask, out, g,
                                      l2_factor, scaled, (T*)dlogits, ld_out, ntok, col0, ncols));
    return check_launch();
}

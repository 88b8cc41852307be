// Grouped GEMM on the 5th-generation tensor cores (tcgen05, kind::f16) with TMA, for the
// dense products around the two hot paths:
//
//   out[m, n] = epi( sum_k A[m, k] W[g, n, k] )     m in rows [offs[g], offs[g+1]) of group g
//
// A (M, K) and W (G, N, K) are row-major fp16 / bf16 (both operands K-major), the group
// offsets live on the device (the launch is sized without reading them on the host, so it
// can be captured in a CUDA graph), fp32 accumulation in tensor memory.  Users:
//   * the full-expert MoE ChannelMix (rwkv_mlx/moe.py:170-242): per expert e, over the rows
//     routed to it, h = relu(x_e @ key_e^T)^2 (epi RELU2) and o = h @ value_e^T (epi STORE);
//   * the output head + l2-wrapped cross-entropy (rwkv_mlx/train.py:317-362): the logits
//     x @ head^T are folded into per-token softmax statistics inside the epilogue (epi CE,
//     each (128-token tile, vocabulary split) keeps its running max / sum / argmax /
//     target logit in registers, so no logit reaches HBM), and the backward recomputes a
//     vocabulary chunk and writes d loss / d logits directly (epi CE_GRAD).
//
// Tiles are 128 rows x 256 columns, K in slices of 64 (one 128-byte swizzle row of a
// 16-bit operand).  The CTA is persistent over work units and warp-specialised:
//   warp 8 lane 0   producer: A and W boxes of each K slice by TMA into a 4-stage ring;
//   warp 9 lane 0   MMA issuer: 4 MMAs (128 x 256 x 16) per slice into one of two
//                   256-column accumulators (tiles alternate), commits to the ring's
//                   "empty" barriers and the accumulator's "full" barrier;
//   warps 0-7       epilogue: TMEM lane 32 (w % 4) + l = row of the tile, warps w and w + 4
//                   take the two 128-column halves; 32 columns per load.
// Logits and outputs are rounded to the activation type before the epilogue uses them,
// as the reference's 16-bit matmul result is.  Every wait is bounded: a wait that gives
// up sets the CTA's abort flag and the device error word, the roles leave their loops,
// the epilogue fills the CTA's remaining outputs with NaN, and the copies and MMAs in
// flight are drained (bounded) before the tensor memory is freed.  No load uses cluster
// multicast.
#include "tma_common.cuh"
#include "wkv7.cuh"

namespace rwkv {

__device__ int g_device_error_gemm;
// Test hook (rwkv_debug_force_wait_timeout): every bounded wait gives up at once.
static __constant__ int c_force_wait_timeout_gemm;

namespace gtc {
using namespace tcc;
using namespace tma;

constexpr int BM = 128, BN = 256, BK = 64, NS = 4;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE = A_BYTES + B_BYTES;
constexpr int NEPI = 256, NTH = NEPI + 64;  // epilogue warps 0-7, producer warp 8, MMA warp 9
constexpr int CTRL = 6144;
constexpr int BAR_EPI = 1;  // named barrier of the epilogue warps
constexpr int MAXG = 256;   // groups per launch
constexpr int SMEM = 1024 /* alignment slack */ + CTRL + NS * STAGE;
static_assert(SMEM <= 227 * 1024, "shared memory");

enum Epi { STORE = 0, RELU2 = 1, CE = 2, CE_GRAD = 3 };

struct Ctrl {
    unsigned long long full[NS], empty[NS], acc_full[2], acc_empty[2], drain;
    uint32_t tmem_base;
    int abort;
    float4 ce_half[BM];  // CE: the second column half's statistics of each row
    int goff[MAXG + 1];  // row offsets of the groups
    int gunit[MAXG + 1]; // first unit of every group; [G] = number of units
};
static_assert(sizeof(Ctrl) <= CTRL, "control block");

struct Args {
    const int32_t* offs;  // G + 1 row offsets, or null: one group of rows [0, M)
    int G, M, N, K;
    int nunit_n;          // units per row tile: N tiles (STORE/RELU2/CE_GRAD) or vocabulary splits (CE)
    int ntn;              // N tiles (ceil(N / BN))
    void* out;            // STORE / RELU2 / CE_GRAD: (M, ldo) in the activation type
    long long ldo;
    int vec_out;          // out rows 16-byte aligned and N % 8 == 0
    // cross-entropy (column col0 + n of the whole vocabulary is column n here)
    const int32_t* targets;
    float4* part;         // CE: (nunit_n, M) partial {max, sum exp(. - max), target logit, argmax}
    const float4* state;  // CE_GRAD: merged {max, sum, target logit, argmax} per token
    const float* mask;    // CE_GRAD: per-token weight or null
    const float* lossout; // CE_GRAD: rwkv_ce_finalize output (den at [3])
    const float* g;       // CE_GRAD: incoming gradient (1 float)
    float l2_factor;
    int scaled;
    int col0;
};

__device__ __forceinline__ bool wait_g(unsigned long long* b, uint32_t parity, volatile int* abort) {
    if (c_force_wait_timeout_gemm) {
        *abort = 1;
        atomicOr(&g_device_error_gemm, 2);
        return false;
    }
    return ck::mbar_wait(b, parity, abort, &g_device_error_gemm);
}
// Bounded wait that ignores the abort flag (draining a role's own copies / MMAs).
__device__ __forceinline__ void drain_wait(unsigned long long* b, uint32_t parity) {
    const uint32_t a = ck::smem_u32(b);
    const long long t0 = clock64();
    while (true) {
        uint32_t ok;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
            : "=r"(ok)
            : "r"(a), "r"(parity)
            : "memory");
        if (ok) return;
        if (clock64() - t0 > ck::WAIT_CYCLES) {
            atomicOr(&g_device_error_gemm, 4);
            return;
        }
    }
}

// Work unit u -> group g, row tile mt of the group, unit j within the row tile.  The
// group table (row offsets and the first unit of every group) is built once per CTA in
// shared memory, so decoding a unit is a short binary search, not a chain of global loads.
struct Unit {
    int g, mt, j, row0, rend;
};
__device__ __forceinline__ Unit unit_of(const Args& p, const int* goff, const int* gunit, int u) {
    int lo = 0, hi = p.G;  // largest g with gunit[g] <= u (empty groups repeat a value)
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (gunit[mid] <= u) lo = mid;
        else hi = mid;
    }
    const int l = u - gunit[lo], mt = l / p.nunit_n;
    return {lo, mt, l % p.nunit_n, goff[lo] + mt * BM, goff[lo + 1]};
}
// N tiles of unit j: one tile, or a contiguous range of tiles (CE vocabulary split).
template <int EPI>
__device__ __forceinline__ void tiles_of(const Args& p, int j, int& t0, int& t1) {
    if (EPI == CE) {
        t0 = (int)((long long)j * p.ntn / p.nunit_n);
        t1 = (int)((long long)(j + 1) * p.ntn / p.nunit_n);
    } else {
        t0 = j, t1 = j + 1;
    }
}

template <typename T>
__device__ __forceinline__ float round_t(float x) {
    return to_f32(from_f32<T>(x));
}

template <typename T>
__device__ __forceinline__ void store32(T* dst, const float* v, int ncol, bool vec) {
    if (vec && ncol >= 32) {
#pragma unroll
        for (int q = 0; q < 32; q += 8) {
            uint4 pk;
            T* pe = reinterpret_cast<T*>(&pk);
#pragma unroll
            for (int e = 0; e < 8; e++) pe[e] = from_f32<T>(v[q + e]);
            *reinterpret_cast<uint4*>(dst + q) = pk;
        }
    } else {
#pragma unroll
        for (int q = 0; q < 32; q++)
            if (q < ncol) dst[q] = from_f32<T>(v[q]);
    }
}

}  // namespace gtc

template <typename T, int EPI>
__global__ void __launch_bounds__(gtc::NTH, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap ma, const __grid_constant__ CUtensorMap mw, const gtc::Args p) {
    using namespace gtc;
    constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
    constexpr uint32_t IDESC = idesc_16(BM, BN, BF, false, false);

    extern __shared__ __align__(1024) unsigned char smem_gtc_raw[];
    const uint32_t raw_addr = ck::smem_u32(smem_gtc_raw);
    unsigned char* smem = smem_gtc_raw + (((raw_addr + 1023) & ~1023u) - raw_addr);
    Ctrl& cs = *reinterpret_cast<Ctrl*>(smem);
    unsigned char* ring = smem + CTRL;  // stage s: A box (16 KB) then W box (32 KB), 1024-aligned
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nk = (p.K + BK - 1) / BK;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                         ck::smem_u32(&cs.tmem_base))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == NEPI) {
        for (int i = 0; i < NS; i++) ck::mbar_init(&cs.full[i], 1), ck::mbar_init(&cs.empty[i], 1);
        for (int i = 0; i < 2; i++) ck::mbar_init(&cs.acc_full[i], 1), ck::mbar_init(&cs.acc_empty[i], NEPI);
        ck::mbar_init(&cs.drain, 1);
        cs.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (tid <= p.G) cs.goff[tid] = p.offs ? p.offs[tid] : (tid == 0 ? 0 : p.M);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) {  // units per group (empty or negative groups: none), exclusive scan over the groups
        constexpr int PER = (MAXG + 31) / 32;
        int loc[PER], sum = 0;
#pragma unroll
        for (int i = 0; i < PER; i++) {
            const int g = lane * PER + i;
            const int rows = g < p.G ? cs.goff[g + 1] - cs.goff[g] : 0;
            loc[i] = sum;
            sum += rows > 0 ? (rows + BM - 1) / BM * p.nunit_n : 0;
        }
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
#pragma unroll
        for (int i = 0; i < PER; i++) {
            const int g = lane * PER + i;
            if (g < p.G) cs.gunit[g] = incl - sum + loc[i];
        }
        if (lane == 31) cs.gunit[p.G] = incl;
    }
    __syncthreads();
    const uint32_t tmem = cs.tmem_base;
    const int nunits = cs.gunit[p.G];

    if (warp == NEPI / 32) {
        // ===================== producer =====================
        if (lane == 0) {
            int it = 0;
            for (int u = blockIdx.x; u < nunits && !*(volatile int*)&cs.abort; u += gridDim.x) {
                const Unit un = unit_of(p, cs.goff, cs.gunit, u);
                int t0, t1;
                tiles_of<EPI>(p, un.j, t0, t1);
                bool bad = false;
                for (int nt = t0; nt < t1 && !bad; nt++) {
                    for (int kb = 0; kb < nk; kb++, it++) {
                        const int s = it % NS;
                        if (it >= NS && !wait_g(&cs.empty[s], ((it / NS) + 1) & 1, &cs.abort)) {
                            bad = true;
                            break;
                        }
                        unsigned char* st = ring + s * STAGE;
                        expect_tx(&cs.full[s], STAGE);
                        tma_load_2d(st, &ma, kb * BK, un.row0, &cs.full[s]);
                        tma_load_3d(st + A_BYTES, &mw, kb * BK, nt * BN, un.g, &cs.full[s]);
                    }
                }
                if (bad) break;
            }
            // the last NS copies may still be in flight: the shared memory they write must
            // stay allocated until they have landed
            for (int i = (it > NS ? it - NS : 0); i < it; i++) drain_wait(&cs.full[i % NS], (i / NS) & 1);
        }
        __syncwarp();
    } else if (warp == NEPI / 32 + 1) {
        // ===================== MMA issuer =====================
        if (lane == 0) {
            int it = 0, q = 0;
            for (int u = blockIdx.x; u < nunits && !*(volatile int*)&cs.abort; u += gridDim.x) {
                const Unit un = unit_of(p, cs.goff, cs.gunit, u);
                int t0, t1;
                tiles_of<EPI>(p, un.j, t0, t1);
                bool bad = false;
                for (int nt = t0; nt < t1 && !bad; nt++, q++) {
                    const int acc = q & 1;
                    if (q >= 2 && !wait_g(&cs.acc_empty[acc], ((q >> 1) + 1) & 1, &cs.abort)) {
                        bad = true;
                        break;
                    }
                    tc_fence_after();
                    for (int kb = 0; kb < nk; kb++, it++) {
                        const int s = it % NS;
                        if (!wait_g(&cs.full[s], (it / NS) & 1, &cs.abort)) {
                            bad = true;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t sa = ck::smem_u32(ring + s * STAGE), sb = sa + A_BYTES;
#pragma unroll
                        for (int kk = 0; kk < BK / 16; kk++)
                            umma16(tmem + acc * BN, desc_sw128(sa + kk * 32, 16, 1024), desc_sw128(sb + kk * 32, 16, 1024),
                                   IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
                        umma_commit(&cs.empty[s]);
                    }
                    if (!bad) umma_commit(&cs.acc_full[acc]);
                }
                if (bad) break;
            }
            if (it > 0) {  // wait for this thread's own MMAs before the memory is freed
                umma_commit(&cs.drain);
                drain_wait(&cs.drain, 0);
            }
        }
        __syncwarp();
    } else {
        // ===================== epilogue =====================
        const int ew = warp & 3, half = warp >> 2;
        const int rl = 32 * ew + lane;  // row of the tile = TMEM lane
        const uint32_t tl = tmem + ((uint32_t)(32 * ew) << 16);
        const int N = p.N;
        bool ab = false;
        int q = 0;
        const float fnan = __int_as_float(0x7fc00000);
        float c1 = 1.f, c2 = 0.f;
        if (EPI == CE_GRAD) {
            const float gv = *p.g, den = p.lossout[3];
            c1 = p.scaled ? gv / den : 1.f;
            c2 = p.scaled ? gv * p.l2_factor : p.l2_factor * den;
        }
        for (int u = blockIdx.x; u < nunits; u += gridDim.x) {
            const Unit un = unit_of(p, cs.goff, cs.gunit, u);
            const int row = un.row0 + rl;
            const bool valid = row >= 0 && row < un.rend && row < p.M;  // (offsets past M are ignored)
            int t0, t1;
            tiles_of<EPI>(p, un.j, t0, t1);
            // CE state of this row over the unit's tiles
            float m = -INFINITY, sum = 0.f, zt = 0.f;
            int am = 0x7fffffff;
            int tg = -1;
            float lse = 0.f, a = 0.f, l2g = 0.f;
            int amg = -1;
            if (EPI == CE && valid) tg = p.targets[row] - p.col0;
            if (EPI == CE_GRAD && valid) {
                const float4 st = p.state[row];
                lse = st.x + logf(st.y);
                a = c1 * (p.mask ? p.mask[row] : 1.f);
                tg = p.targets[row] - p.col0;
                amg = __float_as_int(st.w) - p.col0;
                l2g = c2 * st.x;
            }
            for (int nt = t0; nt < t1; nt++, q++) {
                const int acc = q & 1;
                if (!ab) ab = !wait_g(&cs.acc_full[acc], (q >> 1) & 1, &cs.abort);
                ab = __any_sync(0xffffffffu, ab);
                if (!ab) tc_fence_after();
#pragma unroll 1
                for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += 64) {
                    float vv[2][32];  // two 32-column loads in flight per wait
                    if (!ab) {
                        tmem_ld32(tl + acc * BN + c, vv[0]);
                        tmem_ld32(tl + acc * BN + c + 32, vv[1]);
                        tmem_wait_ld();
                    }
#pragma unroll
                    for (int hh = 0; hh < 2; hh++) {
                        const int n0 = nt * BN + c + 32 * hh;
                        if (n0 >= N || !valid) continue;
                        const int ncol = N - n0 < 32 ? N - n0 : 32;
                        if (EPI == STORE || EPI == RELU2 || EPI == CE_GRAD) {
#pragma unroll
                            for (int e = 0; e < 32; e++) {
                                float x = ab ? fnan : vv[hh][e];
                                if (EPI == RELU2) {
                                    x = round_t<T>(x);  // the key product in the activation type, then relu^2
                                    x = x > 0.f ? x * x : (x == x ? 0.f : x);
                                } else if (EPI == CE_GRAD) {
                                    const float l = round_t<T>(x);
                                    float d = a * (__expf(l - lse) - (n0 + e == tg ? 1.f : 0.f));
                                    if (n0 + e == amg) d += l2g;
                                    x = d;
                                }
                                vv[hh][e] = x;
                            }
                            store32<T>(reinterpret_cast<T*>(p.out) + (size_t)row * p.ldo + n0, vv[hh], ncol, p.vec_out != 0);
                        } else {  // CE
                            if (ab) continue;
                            float lm = -INFINITY;
                            int li = 0;
#pragma unroll
                            for (int e = 0; e < 32; e++) {
                                vv[hh][e] = round_t<T>(vv[hh][e]);
                                if (e < ncol && vv[hh][e] > lm) lm = vv[hh][e], li = e;
                            }
                            if (lm > m) {
                                sum *= __expf(m - lm);
                                m = lm;
                                am = n0 + li;
                            }
#pragma unroll
                            for (int e = 0; e < 32; e++)
                                if (e < ncol) sum += __expf(vv[hh][e] - m);
                            if (tg >= n0 && tg < n0 + ncol) {
#pragma unroll
                                for (int e = 0; e < 32; e++)
                                    if (n0 + e == tg) zt = vv[hh][e];
                            }
                        }
                    }
                }
                if (!ab) {
                    tc_fence_before();
                    ck::mbar_arrive(&cs.acc_empty[acc]);
                }
            }
            if (EPI == CE) {  // merge the two column halves of each row (ties: lower column)
                if (half == 1) cs.ce_half[rl] = make_float4(m, sum, zt, __int_as_float(am));
                ck::bar_sync_n(BAR_EPI, NEPI);
                if (half == 0) {
                    const float4 h1 = cs.ce_half[rl];
                    const int am1 = __float_as_int(h1.w);
                    if (h1.y > 0.f) {
                        if (!(sum > 0.f)) {
                            m = h1.x, sum = h1.y, am = am1;
                        } else if (h1.x > m || (h1.x == m && am1 < am)) {
                            sum = h1.y + sum * __expf(m - h1.x);
                            m = h1.x, am = am1;
                        } else {
                            sum += h1.y * __expf(h1.x - m);
                        }
                    }
                    zt += h1.z;
                    if (valid)
                        p.part[(size_t)un.j * p.M + row] =
                            (ab || *(volatile int*)&cs.abort)
                                ? make_float4(fnan, fnan, fnan, __int_as_float(0x7fffffff))
                                : make_float4(m, sum, zt, __int_as_float(am == 0x7fffffff ? am : am + p.col0));
                }
                ck::bar_sync_n(BAR_EPI, NEPI);  // ce_half is reused by the next unit
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
}

// Merge the CE partials of the vocabulary splits (in column order: ties keep the lower
// column) into the per-token state {max, sum exp(. - max), target logit, argmax}.
__global__ void ce_merge_parts_kernel(const float4* __restrict__ part, int nsplit, int M, float4* __restrict__ state) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= M) return;
    float4 st = part[i];
    for (int s = 1; s < nsplit; s++) {
        const float4 q = part[(size_t)s * M + i];
        if (q.x > st.x) {
            st.y = st.y * __expf(st.x - q.x) + q.y;
            st.x = q.x;
            st.w = q.w;
        } else {
            st.y += q.y * __expf(q.x - st.x);
        }
        st.z += q.z;  // only the split that holds the target contributes
    }
    state[i] = st;
}

namespace gtc {

static int sm_count() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

// Vocabulary splits per 128-token tile for the CE statistics: the smallest count (<= 16,
// <= the N tiles) whose units fill the SMs' last wave to >= 95 %.
static int ce_splits(int M, int ntn) {
    const int mt = (M + BM - 1) / BM, sms = sm_count();
    int best = 1;
    double best_eff = 0.0;
    for (int s = 1; s <= 16 && s <= ntn; s++) {
        const long long u = (long long)mt * s;
        const double eff = (double)u / (double)(((u + sms - 1) / sms) * sms);
        if (eff > best_eff + 1e-9) best = s, best_eff = eff;
        if (eff >= 0.95) return s;
    }
    return best;
}

template <typename T, int EPI>
static int launch(const void* a, const void* w, const Args& p0, int max_units_hint, cudaStream_t st) {
    constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
    Args p = p0;
    p.ntn = (p.N + BN - 1) / BN;
    alignas(64) CUtensorMap ma, mw;
    {  // A (M, K): box 64 x 128 rows, 128-byte swizzle
        const cuuint64_t dims[2] = {(cuuint64_t)p.K, (cuuint64_t)p.M};
        const cuuint64_t strides[1] = {(cuuint64_t)p.K * 2};
        const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)BM};
        const int rc = make_map(&ma, BF, a, 2, dims, strides, box, true);
        if (rc) return RWKV_ERR_CUDA;
    }
    {  // W (G, N, K): box 64 x 256 rows x 1 group, 128-byte swizzle
        const cuuint64_t dims[3] = {(cuuint64_t)p.K, (cuuint64_t)p.N, (cuuint64_t)p.G};
        const cuuint64_t strides[2] = {(cuuint64_t)p.K * 2, (cuuint64_t)p.N * p.K * 2};
        const cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)BN, 1};
        const int rc = make_map(&mw, BF, w, 3, dims, strides, box, true);
        if (rc) return RWKV_ERR_CUDA;
    }
    auto kern = gemm_tc_kernel<T, EPI>;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (err != cudaSuccess) return set_cuda_error(err);
    int grid = sm_count();
    if (max_units_hint > 0 && max_units_hint < grid) grid = max_units_hint;
    kern<<<grid, NTH, SMEM, st>>>(ma, mw, p);
    return check_launch();
}

template <int EPI>
static int dispatch(int dtype, const void* a, const void* w, const Args& p, int hint, cudaStream_t st) {
    switch (dtype) {
        case RWKV_F16: return launch<__half, EPI>(a, w, p, hint, st);
        case RWKV_BF16: return launch<__nv_bfloat16, EPI>(a, w, p, hint, st);
        default: return RWKV_ERR_DTYPE;
    }
}

static int check_common(const void* a, const void* w, int M, int N, int K, int dtype) {
    if (dtype != RWKV_F16 && dtype != RWKV_BF16) return RWKV_ERR_DTYPE;
    if (M <= 0 || N <= 0 || K <= 0 || K % 8) return RWKV_ERR_SHAPE;  // TMA row strides: 16-byte multiples
    if (!a || !w) return RWKV_ERR_ARG;
    if (!aligned(a, 16) || !aligned(w, 16)) return RWKV_ERR_ALIGN;
    return RWKV_OK;
}

}  // namespace gtc

int read_device_error_gemm(int clear) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_error_gemm, sizeof(int));
    if (e != cudaSuccess) return -set_cuda_error(e);
    if (clear && v) {
        const int z = 0;
        e = cudaMemcpyToSymbol(g_device_error_gemm, &z, sizeof(int));
        if (e != cudaSuccess) return -set_cuda_error(e);
    }
    return v;
}
int set_force_wait_timeout_gemm(int on) {
    return set_cuda_error(cudaMemcpyToSymbol(c_force_wait_timeout_gemm, &on, sizeof(int)));
}
int set_device_error_gemm(int value) {
    return set_cuda_error(cudaMemcpyToSymbol(g_device_error_gemm, &value, sizeof(int)));
}

}  // namespace rwkv

using namespace rwkv;

extern "C" int rwkv_grouped_gemm(const void* a, const void* w, const int32_t* offs, void* out, int M, int N, int K,
                                 int G, long long ldo, int epi, int dtype, void* stream) {
    int rc = gtc::check_common(a, w, M, N, K, dtype);
    if (rc) return rc;
    if (G <= 0 || G > gtc::MAXG || (G > 1 && !offs) || !out || ldo < N) return RWKV_ERR_ARG;
    if (epi != gtc::STORE && epi != gtc::RELU2) return RWKV_ERR_ARG;
    gtc::Args p{};
    p.offs = offs, p.G = G, p.M = M, p.N = N, p.K = K;
    p.nunit_n = (N + gtc::BN - 1) / gtc::BN;
    p.out = out, p.ldo = ldo;
    p.vec_out = aligned(out, 16) && (ldo * 2) % 16 == 0 && N % 8 == 0;
    const int hint = offs ? 0 : (M + gtc::BM - 1) / gtc::BM * p.nunit_n;
    cudaStream_t st = (cudaStream_t)stream;
    return epi == gtc::STORE ? gtc::dispatch<gtc::STORE>(dtype, a, w, p, hint, st)
                             : gtc::dispatch<gtc::RELU2>(dtype, a, w, p, hint, st);
}

extern "C" size_t rwkv_head_ce_workspace_size(int M, int V) {
    if (M <= 0 || V <= 0) return 0;
    const int ntn = (V + gtc::BN - 1) / gtc::BN;
    return (size_t)gtc::ce_splits(M, ntn) * M * sizeof(float4);
}

extern "C" int rwkv_head_ce_stats(const void* x, const void* w, const int32_t* targets, float* state, int M, int V,
                                  int K, void* workspace, size_t workspace_bytes, int dtype, void* stream) {
    int rc = gtc::check_common(x, w, M, V, K, dtype);
    if (rc) return rc;
    if (!targets || !state || !workspace) return RWKV_ERR_ARG;
    if (!aligned(state, 16) || !aligned(workspace, 16)) return RWKV_ERR_ALIGN;
    const int ntn = (V + gtc::BN - 1) / gtc::BN, ns = gtc::ce_splits(M, ntn);
    if (workspace_bytes < (size_t)ns * M * sizeof(float4)) return RWKV_ERR_ARG;
    gtc::Args p{};
    p.G = 1, p.M = M, p.N = V, p.K = K;
    p.nunit_n = ns;
    p.targets = targets, p.part = (float4*)workspace;
    cudaStream_t st = (cudaStream_t)stream;
    rc = gtc::dispatch<gtc::CE>(dtype, x, w, p, (M + gtc::BM - 1) / gtc::BM * ns, st);
    if (rc) return rc;
    ce_merge_parts_kernel<<<(M + 255) / 256, 256, 0, st>>>((const float4*)workspace, ns, M, (float4*)state);
    return check_launch();
}

extern "C" int rwkv_head_ce_grad(const void* x, const void* w, const int32_t* targets, const float* state,
                                 const float* mask, const float* out, const float* g, float l2_factor, int scaled,
                                 void* dlogits, long long ld_out, int M, int ncols, int K, int col0, int dtype,
                                 void* stream) {
    int rc = gtc::check_common(x, w, M, ncols, K, dtype);
    if (rc) return rc;
    if (!targets || !state || !out || !g || !dlogits || ld_out < ncols || col0 < 0) return RWKV_ERR_ARG;
    if (!aligned(state, 16)) return RWKV_ERR_ALIGN;
    gtc::Args p{};
    p.G = 1, p.M = M, p.N = ncols, p.K = K;
    p.nunit_n = (ncols + gtc::BN - 1) / gtc::BN;
    p.out = dlogits, p.ldo = ld_out;
    p.vec_out = aligned(dlogits, 16) && (ld_out * 2) % 16 == 0 && ncols % 8 == 0;
    p.targets = targets, p.state = (const float4*)state, p.mask = mask, p.lossout = out, p.g = g;
    p.l2_factor = l2_factor, p.scaled = scaled, p.col0 = col0;
    return gtc::dispatch<gtc::CE_GRAD>(dtype, x, w, p, (M + gtc::BM - 1) / gtc::BM * p.nunit_n, (cudaStream_t)stream);
}

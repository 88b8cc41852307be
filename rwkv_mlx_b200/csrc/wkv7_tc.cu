// WKV-7 forward with the state products on the 5th-generation tensor cores:
// tcgen05.mma (kind::tf32, M=64) with accumulators in tensor memory.  Chunk algebra
// (L = 16; decayed factors as in wkv7_chunk.cu), with Inv = (I - Mab)^-1:
//
//   Wu = Inv At,  Wy = Rt + Mrb Wu,  Gu^T = Inv Mak,  Gy^T = Mrb Gu^T + Mrk,
//   P = Wu^T Bb,  Kb' = Kb + Gu Bb,
//   S_L       = S0 diag(GL) + S0 P + V^T Kb'
//   [U | Y]^T =               S0 [Wu; Wy]^T + V^T [Gu | Gy]
//
// so both right-hand sides are one product with the state, N = 64 + 32 columns, plus
// one with V^T (K = 16).  Per chunk one thread issues 2 + 8 MMAs (a tcgen05.mma keeps
// the tensor pipe ~160 cycles whatever its shape, so the count is what matters) into
// [S_L | U | Y] held in tensor memory; the A operand of the 8 state steps is the fp32
// state itself, read from tensor memory.  The 4 state warps preload S0 diag(GL)
// (exact fp32) and zeros, read S_L back, and store y and sa of the previous chunk
// while the MMAs run.  Two groups of 4 "prep" warps build the inputs-only operands
// for alternating chunks (decay scan, intra-chunk products on mma.sync, forward
// substitution) in the UMMA K-major layout.  Hand-offs are mbarriers with bounded
// waits (a CTA that gives up sets the device error word and exits, it never traps).
//
// Supported for fp16 / bf16 activations (w in the activation dtype or fp32); fp32
// activations use the mma.sync kernel (their input staging does not fit next to this
// kernel's shared memory).
#include <cfloat>

#include "chunk_common.cuh"
#include "common.cuh"
#include "wkv7.cuh"

namespace rwkv {

__device__ int g_device_error_tc;

namespace tc {
using namespace ck;

constexpr int NT = 384;
constexpr int KLBO = 144;  // bytes between K-adjacent core matrices (16 B pad: conflict-free stores)

// byte offset of element (row r, column k) of a K-major no-swizzle UMMA operand
__host__ __device__ constexpr int kmaj(int r, int k, int sbo) {
    return (r & 7) * 16 + (r >> 3) * sbo + (k >> 2) * KLBO + (k & 3) * 4;
}
constexpr int SBO_K64 = 16 * KLBO, SBO_K16 = 4 * KLBO;
constexpr int SZ_BS = 12 * SBO_K64;  // 96 rows x K=64
constexpr int SZ_AV = 8 * SBO_K16;   // 64 rows x K=16
constexpr int SZ_BV = 12 * SBO_K16;  // 96 rows x K=16
constexpr int NS = 96;               // columns of [S_L | U | Y]
constexpr int NSTAGE = 3;            // operand stages (2 prep groups: one chunk of slack)
constexpr uint32_t TMEM_COLS = 256;  // two [S | U | Y] buffers at columns 0 and 128

struct __align__(128) Stage {
    unsigned char BS[SZ_BS];  // B of the state product: rows 0-63 P^T (row j', K = j), 64-79 Wu, 80-95 Wy (K = key)
    unsigned char AV[SZ_AV];  // A of the V product: V^T (row value, K = t)
    unsigned char BV[SZ_BV];  // B of the V product: rows 0-63 Kb'^T (row key), 64-79 Gu^T, 80-95 Gy^T (K = s)
    float GL[N];              // decay of the whole chunk per key
};
struct __align__(16) PrepScratch {
    float At[L][LD4], Rt[L][LD4], Bh[L][LD4], Kh[L][LD4];  // Bh, Kh hold Bb, Kb after P2
    float Mab[L][LDM], Mak[L][LDM], Mrb[L][LDM], Mrk[L][LDM];
    float GuT[L][LDM];
    float Vs[L][LD8];
    float Cs[L + 1][N];  // cumulative log2 decay, Cs[0] = 0
    float GL[N];
};
struct __align__(128) Smem {
    Stage st[NSTAGE];  // chunk c uses stage c % NSTAGE
    float Yb[L][LD8];
    PrepScratch ps[2];
    unsigned long long full[NSTAGE], empty[NSTAGE], mma;
    uint32_t tmem_base;
    int abort;
};

enum { BAR_STATE = 1, BAR_PREP0 = 2 };  // BAR_PREP0 + g for prep group g

// ---- tcgen05 helpers -------------------------------------------------------
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((KLBO >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int Nn) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(Nn >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void umma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p; }" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0)
        : "memory");
}
// same, A (M x K, fp32 columns) read from tensor memory
__device__ __forceinline__ void umma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p; }" ::"r"(d),
        "r"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0)
        : "memory");
}
__device__ __forceinline__ void umma_commit(unsigned long long* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void proxy_fence() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15]))
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void st4(unsigned char* p, float a, float b, float c, float d) {
    *reinterpret_cast<float4*>(p) = make_float4(tf32f(a), tf32f(b), tf32f(c), tf32f(d));
}

// ---------------------------------------------------------------------------
template <typename T, typename TW>
__global__ void __launch_bounds__(NT, 1)
    wkv7_fwd_tc_kernel(const T* __restrict__ r, const TW* __restrict__ w, const T* __restrict__ k,
                       const T* __restrict__ v, const T* __restrict__ a, const T* __restrict__ b,
                       const float* __restrict__ s0, T* __restrict__ y, float* __restrict__ sT,
                       float* __restrict__ ckpt, float* __restrict__ sa_out, int T_, int H,
                       int ckpt_len) {
    using R = Raw<T, TW>;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
    unsigned char* rawbuf = smem_raw + ((sizeof(Smem) + 127) / 128) * 128;  // [2 groups][R::BYTES]

    const int tid = threadIdx.x, warp = tid >> 5;
    const int bh = blockIdx.x, bi = bh / H, hi = bh % H;
    const size_t tstride = (size_t)H * N;
    const size_t base = ((size_t)bi * T_ * H + hi) * N;
    const int nchunks = (T_ + L - 1) / L;
    const int nck = ckpt ? T_ / ckpt_len : 0;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&sm.tmem_base)), "n"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 32) {
        for (int i = 0; i < NSTAGE; i++) {
            mbar_init(&sm.full[i], 128);
            mbar_init(&sm.empty[i], 128);
        }
        mbar_init(&sm.mma, 1);
        sm.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;

    if (warp >= 4) {
        // ===================== prep groups: chunks g_, g_ + 2, ... into stage g_ =====================
        const int g_ = (warp - 4) >> 2;
        const int pt = tid - 128 - 128 * g_, pw = pt >> 5, lane = pt & 31, g = lane >> 2, tg = lane & 3;
        const int BAR = BAR_PREP0 + g_;
        PrepScratch& ps = sm.ps[g_];
        unsigned char* raw = rawbuf + (size_t)g_ * R::BYTES;

        const char* psrc[R::PER_THREAD];
        uint32_t pdst[R::PER_THREAD];
        int prow[R::PER_THREAD];
#pragma unroll
        for (int i = 0; i < R::PER_THREAD; i++) {
            const int q = pt + 128 * i;
            if (q < 5 * L * R::PPR) {
                const int arr = q / (L * R::PPR), rem = q % (L * R::PPR), row = rem / R::PPR, pc = rem % R::PPR;
                const T* src = arr == 0 ? r : arr == 1 ? k : arr == 2 ? v : arr == 3 ? a : b;
                psrc[i] = reinterpret_cast<const char*>(src + base + (size_t)row * tstride) + pc * 16;
                pdst[i] = arr * R::ARR + row * R::PITCH + pc * 16;
                prow[i] = row;
            } else if (q < R::PIECES) {
                const int q2 = q - 5 * L * R::PPR, row = q2 / R::PPRW, pc = q2 % R::PPRW;
                psrc[i] = reinterpret_cast<const char*>(w + base + (size_t)row * tstride) + pc * 16;
                pdst[i] = 5 * R::ARR + row * R::PITCHW + pc * 16;
                prow[i] = row;
            } else {
                psrc[i] = nullptr, pdst[i] = 0, prow[i] = -1;
            }
        }
        auto issue = [&](int c) {
            const int t0 = c * L;
#pragma unroll
            for (int i = 0; i < R::PER_THREAD; i++) {
                if (prow[i] < 0) continue;
                const bool ok = (t0 + prow[i]) < T_;
                const size_t step = (size_t)t0 * tstride;
                const char* src = ok ? psrc[i] + step * (pdst[i] >= 5u * R::ARR ? sizeof(TW) : sizeof(T)) : psrc[i];
                cp_async16(raw + pdst[i], src, ok);
            }
            cp_commit();
        };
        auto ldB = [&](const unsigned char* src, int kk, int nn) {
            return fbits(*reinterpret_cast<const float*>(src + kmaj(kk, nn, SBO_K64)));
        };

        if (g_ < nchunks) issue(g_);
        for (int c = g_; c < nchunks; c += 2) {
            asm volatile("cp.async.wait_all;" ::: "memory");
            group_sync(BAR);

            // ---- P1: cumulative log2 decay, decayed factors ----
            const int t = lane & 15, cg = 2 * pw + (lane >> 4), j0 = 8 * cg;
            const bool tok = t < T_ - c * L;
            float wv[8], cs[8], cl[8], ec[8], ei[8], ep[8];
            lds8<TW>(raw + 5 * R::ARR + t * R::PITCHW + j0 * sizeof(TW), wv);
#pragma unroll
            for (int q = 0; q < 8; q++) cs[q] = tok ? -ex2(wv[q] * LOG2E) * LOG2E : 0.f;
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) {
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    const float u = __shfl_up_sync(0xffffffffu, cs[q], o, 16);
                    if (t >= o) cs[q] += u;
                }
            }
            bool ext = false;
#pragma unroll
            for (int q = 0; q < 8; q++) {
                ec[q] = ex2(cs[q]);
                ei[q] = ex2(-cs[q]);
                cl[q] = __shfl_sync(0xffffffffu, cs[q], 15, 16);
                const float up = __shfl_up_sync(0xffffffffu, ec[q], 1, 16);
                ep[q] = t ? up : 1.f;
                ext |= cl[q] < -115.f;  // cumulative decay below e^-80
            }
            float bb[8], kb[8];
            {
                float xr[8], xk[8], xv[8], xa[8], xb[8], o1[8], o2[8];
                lds8<T>(raw + 0 * R::ARR + t * R::PITCH + j0 * sizeof(T), xr);
                lds8<T>(raw + 1 * R::ARR + t * R::PITCH + j0 * sizeof(T), xk);
                lds8<T>(raw + 2 * R::ARR + t * R::PITCH + j0 * sizeof(T), xv);
                lds8<T>(raw + 3 * R::ARR + t * R::PITCH + j0 * sizeof(T), xa);
                lds8<T>(raw + 4 * R::ARR + t * R::PITCH + j0 * sizeof(T), xb);
#pragma unroll
                for (int q = 0; q < 8; q++) o1[q] = tf32f(xa[q] * ep[q]), o2[q] = tf32f(xr[q] * ec[q]);
                sts8(&ps.At[t][j0], o1);
                sts8(&ps.Rt[t][j0], o2);
#pragma unroll
                for (int q = 0; q < 8; q++) o1[q] = tf32f(xb[q] * ei[q]), o2[q] = tf32f(xk[q] * ei[q]);
                sts8(&ps.Bh[t][j0], o1);
                sts8(&ps.Kh[t][j0], o2);
                // factors to the chunk end: 2^(cL - c_t) (the product form overflows only
                // where the chunk's decay is extreme; those keys take the direct form)
                float eL[8];
#pragma unroll
                for (int q = 0; q < 8; q++) eL[q] = __shfl_sync(0xffffffffu, ec[q], 15, 16) * ei[q];
                if (ext) {
#pragma unroll
                    for (int q = 0; q < 8; q++) eL[q] = ex2(cl[q] - cs[q]);
                }
#pragma unroll
                for (int q = 0; q < 8; q++) bb[q] = tf32f(xb[q] * eL[q]), kb[q] = tf32f(xk[q] * eL[q]), o1[q] = tf32f(xv[q]);
                sts8(&ps.Vs[t][j0], o1);
            }
            sts8(&ps.Cs[t + 1][j0], cs);
            if (t == 0) {
#pragma unroll
                for (int q = 0; q < 8; q++) ps.Cs[0][j0 + q] = 0.f;
            }
            if (t == 15) sts8(&ps.GL[j0], ec);
            const bool extreme = group_sync_or(BAR, ext);

            // ---- P2: intra-chunk matrices ----
            if (!extreme) {
                const float(*Am)[LD4] = (pw >> 1) ? ps.Rt : ps.At;
                const float(*Bm)[LD4] = (pw & 1) ? ps.Kh : ps.Bh;
                float acc2[2][4] = {};
#pragma unroll
                for (int ks = 0; ks < 8; ks++) {
                    const int k0 = 8 * ks;
                    const uint32_t a0 = fbits(Am[g][k0 + tg]), a1 = fbits(Am[g + 8][k0 + tg]);
                    const uint32_t a2 = fbits(Am[g][k0 + tg + 4]), a3 = fbits(Am[g + 8][k0 + tg + 4]);
#pragma unroll
                    for (int nt = 0; nt < 2; nt++) {
                        const uint32_t b0 = fbits(Bm[8 * nt + g][k0 + tg]), b1 = fbits(Bm[8 * nt + g][k0 + tg + 4]);
                        mma8(acc2[nt], a0, a1, a2, a3, b0, b1);
                    }
                }
                float(*Mo)[LDM] = pw == 0 ? ps.Mab : pw == 1 ? ps.Mak : pw == 2 ? ps.Mrb : ps.Mrk;
                const bool strict = pw < 2;
#pragma unroll
                for (int nt = 0; nt < 2; nt++) {
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int tt = g + (e >> 1) * 8, sidx = 8 * nt + 2 * tg + (e & 1);
                        const bool keep = strict ? (sidx < tt) : (sidx <= tt);
                        const float val = keep ? acc2[nt][e] : 0.f;
                        Mo[tt][sidx] = (pw == 0) ? val : tf32f(val);
                    }
                }
            } else {
                for (int e = pt; e < 4 * L * L; e += 128) {
                    const int which = e / (L * L), tt = (e / L) % L, sidx = e % L;
                    const bool strict = which < 2;
                    float val = 0.f;
                    if (strict ? (sidx < tt) : (sidx <= tt)) {
                        const T* lhs = reinterpret_cast<const T*>(raw + (which < 2 ? 3 : 0) * R::ARR + tt * R::PITCH);
                        const T* rhs = reinterpret_cast<const T*>(raw + ((which & 1) ? 1 : 4) * R::ARR + sidx * R::PITCH);
                        const float* cl2 = (which < 2) ? ps.Cs[tt] : ps.Cs[tt + 1];
                        const float* cr2 = ps.Cs[sidx + 1];
                        for (int jj = 0; jj < N; jj++)
                            val = fmaf(to_f32(lhs[jj]) * to_f32(rhs[jj]), exp2f(cl2[jj] - cr2[jj]), val);
                    }
                    float(*Mo)[LDM] = which == 0 ? ps.Mab : which == 1 ? ps.Mak : which == 2 ? ps.Mrb : ps.Mrk;
                    Mo[tt][sidx] = which == 0 ? val : tf32f(val);
                }
            }
            group_sync(BAR);
            if (c + 2 < nchunks) issue(c + 2);  // raw staging is free from here on
            sts8(&ps.Bh[t][j0], bb);           // Bh, Kh are dead: keep Bb, Kb there
            sts8(&ps.Kh[t][j0], kb);

            // ---- P4: forward substitution (I - Mab) X = [At | Mak]: Wu (threads 0-63, one key
            //      column each) and Gu^T (threads 64-79, one column each), column-oriented
            const int col = pt;
            float x[L];
            if (pt < N + L) {
#pragma unroll
                for (int tt = 0; tt < L; tt++) x[tt] = pt < N ? ps.At[tt][col] : ps.Mak[tt][col - N];
#pragma unroll
                for (int s2 = 0; s2 < L - 1; s2++) {
#pragma unroll
                    for (int tt = s2 + 1; tt < L; tt++) x[tt] = fmaf(ps.Mab[tt][s2], x[s2], x[tt]);
                }
                if (pt >= N) {
#pragma unroll
                    for (int tt = 0; tt < L; tt++) ps.GuT[tt][col - N] = tf32f(x[tt]);
                }
            }

            // ---- the stage is free once the state warps are done with chunk c - 2 ----
            bool bad = false;
            const int si = c % NSTAGE;
            Stage& stg = sm.st[si];
            if (c >= NSTAGE) bad = !mbar_wait(&sm.empty[si], ((c / NSTAGE) + 1) & 1, &sm.abort, &g_device_error_tc);
            if (group_sync_or(BAR, bad)) break;

            // ---- B1: Wu -> BS rows 64-79, V^T -> AV, GL ----
            if (pt < N) {
#pragma unroll
                for (int tt = 0; tt < L; tt++) *reinterpret_cast<float*>(stg.BS + kmaj(N + tt, col, SBO_K64)) = tf32f(x[tt]);
#pragma unroll
                for (int tt = 0; tt < L; tt += 4)
                    *reinterpret_cast<float4*>(stg.AV + kmaj(col, tt, SBO_K16)) =
                        make_float4(ps.Vs[tt][col], ps.Vs[tt + 1][col], ps.Vs[tt + 2][col], ps.Vs[tt + 3][col]);
            } else {
                stg.GL[pt - N] = ps.GL[pt - N];
            }
            group_sync(BAR);

            // ---- B2: Wy = Rt + Mrb Wu -> BS rows 80-95; P^T -> BS rows 0-63;
            //      Kb'^T -> BV rows 0-63; Gu^T, Gy^T -> BV rows 64-95 ----
            {
                float wy[2][4];
#pragma unroll
                for (int nt = 0; nt < 2; nt++) {
                    const int n0 = 16 * pw + 8 * nt + 2 * tg;
                    wy[nt][0] = ps.Rt[g][n0], wy[nt][1] = ps.Rt[g][n0 + 1];
                    wy[nt][2] = ps.Rt[g + 8][n0], wy[nt][3] = ps.Rt[g + 8][n0 + 1];
                }
#pragma unroll
                for (int ks = 0; ks < 2; ks++) {
                    const int k0 = 8 * ks;
                    const uint32_t a0 = fbits(ps.Mrb[g][k0 + tg]), a1 = fbits(ps.Mrb[g + 8][k0 + tg]);
                    const uint32_t a2 = fbits(ps.Mrb[g][k0 + tg + 4]), a3 = fbits(ps.Mrb[g + 8][k0 + tg + 4]);
#pragma unroll
                    for (int nt = 0; nt < 2; nt++) {
                        const int n0 = 16 * pw + 8 * nt;
                        mma8(wy[nt], a0, a1, a2, a3, ldB(stg.BS, N + k0 + tg, n0 + g), ldB(stg.BS, N + k0 + tg + 4, n0 + g));
                    }
                }
#pragma unroll
                for (int nt = 0; nt < 2; nt++) {
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int tt = N + L + g + (e >> 1) * 8, cc = 16 * pw + 8 * nt + 2 * tg + (e & 1);
                        *reinterpret_cast<float*>(stg.BS + kmaj(tt, cc, SBO_K64)) = tf32f(wy[nt][e]);
                    }
                }
            }
            {
                // P[j][j'] = sum_t Wu[t][j] Bb[t][j']; row j' (= 16 pw + ...) of the K-major operand
                float pl[8][4] = {};
                const int m0 = 16 * pw;
#pragma unroll
                for (int ks = 0; ks < 2; ks++) {
                    const int k0 = 8 * ks;
                    const uint32_t a0 = fbits(ps.Bh[k0 + tg][m0 + g]), a1 = fbits(ps.Bh[k0 + tg][m0 + g + 8]);
                    const uint32_t a2 = fbits(ps.Bh[k0 + tg + 4][m0 + g]), a3 = fbits(ps.Bh[k0 + tg + 4][m0 + g + 8]);
#pragma unroll
                    for (int nt = 0; nt < 8; nt++)
                        mma8(pl[nt], a0, a1, a2, a3, ldB(stg.BS, N + k0 + tg, 8 * nt + g), ldB(stg.BS, N + k0 + tg + 4, 8 * nt + g));
                }
#pragma unroll
                for (int nt = 0; nt < 8; nt++) {
                    const int jj = 8 * nt + 2 * tg;
                    *reinterpret_cast<float2*>(stg.BS + kmaj(m0 + g, jj, SBO_K64)) = make_float2(tf32f(pl[nt][0]), tf32f(pl[nt][1]));
                    *reinterpret_cast<float2*>(stg.BS + kmaj(m0 + g + 8, jj, SBO_K64)) = make_float2(tf32f(pl[nt][2]), tf32f(pl[nt][3]));
                }
            }
            {
                // Kb'[s][j] = Kb[s][j] + sum_t' Gu^T[t'][s] Bb[t'][j] for keys j in [16 pw, 16 pw + 16)
                float kq[2][4];
#pragma unroll
                for (int nt = 0; nt < 2; nt++) {
                    const int n0 = 16 * pw + 8 * nt + 2 * tg;
                    kq[nt][0] = ps.Kh[g][n0], kq[nt][1] = ps.Kh[g][n0 + 1];
                    kq[nt][2] = ps.Kh[g + 8][n0], kq[nt][3] = ps.Kh[g + 8][n0 + 1];
                }
#pragma unroll
                for (int ks = 0; ks < 2; ks++) {
                    const int k0 = 8 * ks;
                    const uint32_t a0 = fbits(ps.GuT[k0 + tg][g]), a1 = fbits(ps.GuT[k0 + tg][g + 8]);
                    const uint32_t a2 = fbits(ps.GuT[k0 + tg + 4][g]), a3 = fbits(ps.GuT[k0 + tg + 4][g + 8]);
#pragma unroll
                    for (int nt = 0; nt < 2; nt++) {
                        const int n0 = 16 * pw + 8 * nt;
                        mma8(kq[nt], a0, a1, a2, a3, fbits(ps.Bh[k0 + tg][n0 + g]), fbits(ps.Bh[k0 + tg + 4][n0 + g]));
                    }
                }
#pragma unroll
                for (int nt = 0; nt < 2; nt++) {
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int ss = g + (e >> 1) * 8, jj = 16 * pw + 8 * nt + 2 * tg + (e & 1);
                        *reinterpret_cast<float*>(stg.BV + kmaj(jj, ss, SBO_K16)) = tf32f(kq[nt][e]);
                    }
                }
            }
            if (pw == 0) {
                // Gy^T[t'][s] = sum_u Mrb[t'][u] Gu^T[u][s] + Mrk[t'][s]
                float gy[2][4];
#pragma unroll
                for (int nt = 0; nt < 2; nt++) {
                    const int n0 = 8 * nt + 2 * tg;
                    gy[nt][0] = ps.Mrk[g][n0], gy[nt][1] = ps.Mrk[g][n0 + 1];
                    gy[nt][2] = ps.Mrk[g + 8][n0], gy[nt][3] = ps.Mrk[g + 8][n0 + 1];
                }
#pragma unroll
                for (int ks = 0; ks < 2; ks++) {
                    const int k0 = 8 * ks;
                    const uint32_t a0 = fbits(ps.Mrb[g][k0 + tg]), a1 = fbits(ps.Mrb[g + 8][k0 + tg]);
                    const uint32_t a2 = fbits(ps.Mrb[g][k0 + tg + 4]), a3 = fbits(ps.Mrb[g + 8][k0 + tg + 4]);
#pragma unroll
                    for (int nt = 0; nt < 2; nt++)
                        mma8(gy[nt], a0, a1, a2, a3, fbits(ps.GuT[k0 + tg][8 * nt + g]), fbits(ps.GuT[k0 + tg + 4][8 * nt + g]));
                }
#pragma unroll
                for (int nt = 0; nt < 2; nt++) {
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int tp = g + (e >> 1) * 8, ss = 8 * nt + 2 * tg + (e & 1);
                        *reinterpret_cast<float*>(stg.BV + kmaj(N + L + tp, ss, SBO_K16)) = tf32f(gy[nt][e]);
                    }
                }
            } else if (pw == 1) {
#pragma unroll
                for (int i = 0; i < (L * L) / 32; i++) {
                    const int q = lane + 32 * i, tp = q / L, ss = q % L;
                    *reinterpret_cast<float*>(stg.BV + kmaj(N + tp, ss, SBO_K16)) = ps.GuT[tp][ss];
                }
            }

            // ---- B3: hand the chunk over ----
            proxy_fence();  // operand stores -> async proxy
            mbar_arrive(&sm.full[si]);
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else {
        // ===================== state warps =====================
        // tensor memory: buffer b at column 128 b holds [S (64) | U (16) | Y (16)]; chunk c
        // reads the state from buffer c & 1 and accumulates into buffer (c + 1) & 1
        const int tw = warp, lane = tid & 31;
        const bool live = lane < 16;              // M=64 accumulators use lanes 0-15 of each subpartition
        const int row = 16 * tw + lane;            // state row (value index) held by this thread
        const uint32_t tl = tmem + ((uint32_t)(32 * tw) << 16);
        auto buf = [](int c) { return (uint32_t)(128 * (c & 1)); };

        // y and sa of chunk cc from its buffer (U at +64, Y at +80)
        auto output = [&](int cc) {
            float u[L], yv[L];
            const uint32_t d = tl + buf(cc + 1) + N;
            tmem_ld16(d, u);
            tmem_ld16(d + L, yv);
            tmem_wait_ld();
            if (live) {
#pragma unroll
                for (int tt = 0; tt < L; tt++) sm.Yb[tt][row] = yv[tt];
                if (sa_out) {
#pragma unroll
                    for (int tt = 0; tt < L; tt++)
                        if (cc * L + tt < T_) sa_out[base + (size_t)(cc * L + tt) * tstride + row] = u[tt];
                }
            }
            group_sync(BAR_STATE);
            const int rr = tid >> 3, c8 = (tid & 7) * 8, t = cc * L + rr;
            if (t < T_) {
                const float4 f0 = *reinterpret_cast<const float4*>(&sm.Yb[rr][c8]);
                const float4 f1 = *reinterpret_cast<const float4*>(&sm.Yb[rr][c8 + 4]);
                uint4 pk;
                T* pe = reinterpret_cast<T*>(&pk);
                pe[0] = from_f32<T>(f0.x), pe[1] = from_f32<T>(f0.y), pe[2] = from_f32<T>(f0.z), pe[3] = from_f32<T>(f0.w);
                pe[4] = from_f32<T>(f1.x), pe[5] = from_f32<T>(f1.y), pe[6] = from_f32<T>(f1.z), pe[7] = from_f32<T>(f1.w);
                *reinterpret_cast<uint4*>(y + base + (size_t)t * tstride + c8) = pk;
            }
        };
        // S (state after chunk cn - 1, from tensor memory or s0) -> checkpoint when due;
        // S diag(GL of chunk cn) and zero [U | Y] -> buffer (cn + 1) & 1
        auto advance = [&](int cn, bool have_next, bool from_s0) {
            const int tend = cn * L;
            const bool save = ckpt && cn > 0 && tend <= T_ && tend % ckpt_len == 0;
            const Stage& stg = sm.st[cn % NSTAGE];
            const uint32_t from = tl + buf(cn), to = tl + buf(cn + 1);
#pragma unroll
            for (int h = 0; h < 2; h++) {
                float S[32];
                if (from_s0) {
                    const float* p = (s0 && live) ? s0 + ((size_t)bh * N + row) * N + 32 * h : nullptr;
#pragma unroll
                    for (int j = 0; j < 32; j++) S[j] = p ? p[j] : 0.f;
                    tmem_st16(from + 32 * h, S);
                    tmem_st16(from + 32 * h + 16, S + 16);
                } else {
                    tmem_ld16(from + 32 * h, S);
                    tmem_ld16(from + 32 * h + 16, S + 16);
                    tmem_wait_ld();
                }
                if (save && live) {
                    float* p = ckpt + (((size_t)bh * nck + tend / ckpt_len - 1) * N + row) * N + 32 * h;
#pragma unroll
                    for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(p + j) = make_float4(S[j], S[j + 1], S[j + 2], S[j + 3]);
                }
                if (have_next) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        const float4 gl = *reinterpret_cast<const float4*>(&stg.GL[32 * h + j]);
                        S[j] *= gl.x, S[j + 1] *= gl.y, S[j + 2] *= gl.z, S[j + 3] *= gl.w;
                    }
                    tmem_st16(to + 32 * h, S);
                    tmem_st16(to + 32 * h + 16, S + 16);
                }
            }
            if (have_next) {
                float z[16];
#pragma unroll
                for (int j = 0; j < 16; j++) z[j] = 0.f;
                tmem_st16(to + N, z);
                tmem_st16(to + N + L, z);
            }
            tmem_wait_st();
        };

        bool ok = true;
        if (nchunks > 0) {
            ok = !group_sync_or(BAR_STATE, !mbar_wait(&sm.full[0], 0, &sm.abort, &g_device_error_tc));
            advance(0, ok, true);  // s0 -> buffer 0; S0 diag(GL) and zeros -> buffer 1
        } else {
            advance(0, false, true);
        }
        for (int c = 0; ok && c < nchunks; c++) {
            tc_fence_before();
            group_sync(BAR_STATE);
            tc_fence_after();
            if (tid == 0) {
                const Stage& stg = sm.st[c % NSTAGE];
                const uint32_t id = idesc_tf32(64, NS);
                const uint32_t aV = smem_u32(stg.AV), bV = smem_u32(stg.BV), bS = smem_u32(stg.BS);
                const uint32_t d = tmem + buf(c + 1), a_ = tmem + buf(c);
#pragma unroll
                for (int ks = 0; ks < 2; ks++)
                    umma(d, umma_desc(aV + 2 * ks * KLBO, SBO_K16), umma_desc(bV + 2 * ks * KLBO, SBO_K16), id, 1);
#pragma unroll
                for (int ks = 0; ks < 8; ks++)
                    umma_ts(d, a_ + 8 * ks, umma_desc(bS + 2 * ks * KLBO, SBO_K64), id, 1);
                umma_commit(&sm.mma);
            }
            if (c >= 1) output(c - 1);
            const bool more = c + 1 < nchunks;
            bool bad = more && !mbar_wait(&sm.full[(c + 1) % NSTAGE], ((c + 1) / NSTAGE) & 1, &sm.abort, &g_device_error_tc);
            bad |= !mbar_wait(&sm.mma, c & 1, &sm.abort, &g_device_error_tc);
            tc_fence_after();
            advance(c + 1, more, false);
            tc_fence_before();
            mbar_arrive(&sm.empty[c % NSTAGE]);
            ok = !group_sync_or(BAR_STATE, bad);  // uniform decision for the whole group
        }
        if (ok && nchunks > 0) output(nchunks - 1);
        if (sT && ok) {
            const uint32_t fin = tl + buf(nchunks);
#pragma unroll
            for (int h = 0; h < 2; h++) {
                float S[32];
                tmem_ld16(fin + 32 * h, S);
                tmem_ld16(fin + 32 * h + 16, S + 16);
                tmem_wait_ld();
                if (live) {
                    float* p = sT + ((size_t)bh * N + row) * N + 32 * h;
#pragma unroll
                    for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(p + j) = make_float4(S[j], S[j + 1], S[j + 2], S[j + 3]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(TMEM_COLS) : "memory");
    }
}

template <typename T, typename TW>
size_t smem_bytes() {
    return ((sizeof(Smem) + 127) / 128) * 128 + 2 * (size_t)Raw<T, TW>::BYTES;
}

}  // namespace tc

template <typename T, typename TW>
static int launch_fwd_tc(const WkvFwdArgs& p, cudaStream_t st) {
    auto kern = tc::wkv7_fwd_tc_kernel<T, TW>;
    const size_t smem = tc::smem_bytes<T, TW>();
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_cuda_error(e);
    kern<<<p.B * p.H, tc::NT, smem, st>>>((const T*)p.r, (const TW*)p.w, (const T*)p.k, (const T*)p.v,
                                          (const T*)p.a, (const T*)p.b, p.s0, (T*)p.y, p.sT, p.ckpt, p.sa,
                                          p.T, p.H, p.ckpt_len);
    return check_launch();
}

bool wkv7_tc_supported(int dtype) { return dtype == RWKV_F16 || dtype == RWKV_BF16; }

int wkv7_fwd_tc(const WkvFwdArgs& p, cudaStream_t st) {
    switch (p.dtype) {
        case RWKV_F16:
            if (p.w_dtype == RWKV_F16) return launch_fwd_tc<__half, __half>(p, st);
            if (p.w_dtype == RWKV_F32) return launch_fwd_tc<__half, float>(p, st);
            return RWKV_ERR_DTYPE;
        case RWKV_BF16:
            if (p.w_dtype == RWKV_BF16) return launch_fwd_tc<__nv_bfloat16, __nv_bfloat16>(p, st);
            if (p.w_dtype == RWKV_F32) return launch_fwd_tc<__nv_bfloat16, float>(p, st);
            return RWKV_ERR_DTYPE;
        default:
            return RWKV_ERR_DTYPE;
    }
}

int read_device_error_tc(int clear) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_error_tc, sizeof(int));
    if (e != cudaSuccess) return -set_cuda_error(e);
    if (clear && v) {
        const int z = 0;
        e = cudaMemcpyToSymbol(g_device_error_tc, &z, sizeof(int));
        if (e != cudaSuccess) return -set_cuda_error(e);
    }
    return v;
}

}  // namespace rwkv

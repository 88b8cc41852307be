// WKV-7 forward with the state products on the 5th-generation tensor cores:
// tcgen05.mma (kind::tf32) with accumulators in tensor memory.  Same chunk algebra as
// wkv7_chunk.cu (L = 16 steps per chunk, S0 the state entering the chunk):
//
//   U^T = S0 Wu^T + Ui^T,  Y^T = S0 Wy^T + Yi^T               (sa and y of the chunk)
//   S_L = S0 diag(GL) + V^T Kb + U^T Bb
//
// with the inputs-only parts Ui^T = V^T Gu, Yi^T = V^T Gy and V^T Kb formed as one
// product X = V^T [Gu | Gy | Kb] (N = 96).
//
// Cost model (measured on B200): a tcgen05.mma blocks the thread that issues it for
// ~280 cycles with A in shared memory and ~165 with A in tensor memory, whatever its
// shape, while separate warps issue in parallel.  The serial state chain is therefore
// arranged around MMA issues, not FLOPs:
//   * the K = 64 product S0 [Wu; Wy]^T is split over the 4 state warps: warp w issues
//     the two K-steps of keys 16w..16w+15 into its own accumulator D1_w (A = the state
//     read from tensor memory), so the chain pays for 2 issues instead of 8;
//   * X, which needs no state, is issued by the prep group that built the chunk (its
//     completion is part of the chunk's "full" barrier), off the chain;
//   * the state warps sum U = sum_w D1_w.u + X.u, write it to tensor memory, form
//     S0 diag(GL) + V^T Kb in registers (one read-modify-write of the state), and one
//     thread issues U^T Bb with A = U read from tensor memory (2 issues).
// Two groups of 4 "prep" warps compute the inputs-only chunk operands (decay scan,
// intra-chunk products on mma.sync, triangular solve) for alternating chunks, straight
// into the UMMA operand layouts; each group's six input boxes (16 steps of r, k, v, a, b,
// w) arrive by TMA one own chunk ahead, issued by one thread.  Every wait is a bounded mbarrier wait: a CTA that
// gives up sets the device error word, waits (bounded) for its own MMAs in flight,
// fills its outputs with NaN, frees its tensor memory and exits; it never traps.
//
// Segments (intra-sequence parallelism for small B*H): the sequence is cut into nseg
// segments of whole chunks.  A "transition" launch runs each segment s < nseg-1 with a
// 128-row state [C; M] (C from S = 0, or from s0 for segment 0; M from the identity,
// no inputs), which gives the segment's affine map S_end = S_start M + C at the cost
// of the 64-row chain (MMA issues do not depend on M).  wkv7_seg_scan_kernel composes
// the maps into every segment's initial state, and the forward launch runs all
// segments in parallel from those states.
//
// Supported for fp16 / bf16 activations (w in the activation dtype or fp32); fp32
// activations use the mma.sync kernel.
#include <cfloat>

#include "chunk_common.cuh"
#include "common.cuh"
#include "tc_common.cuh"
#include "tma_common.cuh"
#include "wkv7.cuh"
#include "wkv_stage.cuh"

namespace rwkv {

__device__ int g_device_error_tc;
// Test hook (rwkv_debug_force_wait_timeout): every bounded wait of these kernels gives
// up at once, which exercises the abort path without any real stall.
static __constant__ int c_force_wait_timeout;

namespace tc {
using namespace ck;
using namespace tcc;
using namespace tma;

constexpr int NT = 384;
constexpr int NSTAGE = 3;  // operand stages for 2 prep groups: one chunk of slack
constexpr int SBO_K64 = 16 * KLBO, SBO_K16 = 4 * KLBO;
constexpr int SZ_WB = 4 * SBO_K64;   // 32 rows x K=64
constexpr int SZ_BB = 8 * SBO_K16;   // 64 rows x K=16
constexpr int SZ_BX = 12 * SBO_K16;  // 96 rows x K=16

// Tensor-memory columns: state, the four D1 partial products, U, X per stage.
constexpr uint32_t COL_S = 0, COL_D1 = 64, COL_U = 192, COL_X = 208;
constexpr int ROWS_CM = 128;  // rows of a segment's transition output [C; M]

template <int ROWS>
struct __align__(128) Stage {
    unsigned char WB[SZ_WB];                  // B of D1: rows t' (0-15 Wu, 16-31 Wy), K = key
    unsigned char BB[SZ_BB];                  // B of U^T Bb: rows key, K = t
    unsigned char BX[SZ_BX];                  // B of X: rows 0-15 Gu^T, 16-31 Gy^T, 32-95 Kb (key), K = s
    unsigned char VT[(ROWS / 8) * SBO_K16];   // A of X: rows value (>= 64: zero), K = t
    float GL[N];                              // decay of the whole chunk per key
};
struct __align__(16) PrepScratch {
    float At[L][LD4], Rt[L][LD4], Bh[L][LD4], Kh[L][LD4];
    float Mab[L][LDM], Mak[L][LDM], Mrb[L][LDM], Mrk[L][LDM];
    float GuT[L][LDM];  // (I - Mab)^-1 Mak
    float Cs[L + 1][LD4];  // cumulative log2 decay, Cs[0] = 0 (rows padded: conflict-free stores)
};
template <int ROWS>
struct __align__(128) Smem {
    Stage<ROWS> st[NSTAGE];  // chunk c uses stage c % NSTAGE
    float Yb[L][LD8];
    PrepScratch ps[2];
    unsigned long long full[NSTAGE], empty[NSTAGE], mma1, mma2, drain[3];
    unsigned long long ld_full[2];  // a prep group's input staging has landed (TMA)
    uint32_t tmem_base;
    int abort;
};

// Input staging of one prep group (one TMA box per array, wkv_stage.cuh): r, k, v, a, b,
// then w.
template <typename T, typename TW>
struct RawT {
    static constexpr int ARR = wst::box_bytes<T>();
    static constexpr int BYTES = 5 * ARR + wst::box_bytes<TW>();  // a multiple of 1024
};
using wst::InMaps;

enum { BAR_STATE = 1, BAR_PREP0 = 2 };  // BAR_PREP0 + g for prep group g

struct TcArgs {
    const void *r, *w, *k, *v, *a, *b;
    const float* s0;  // initial state of the sequence (B,H,64,64) or null
    void* y;
    float *sT, *ckpt, *sa;
    float* seg_s0;  // forward launch, nseg > 1: state entering segment s >= 1, ((bh*nseg+s)*64+row)*64
    float* trans;   // transition launch: [C; M] of segment s < nseg-1, ((bh*(nseg-1)+s)*128+row)*64
    int T, H, ckpt_len, nseg, seg_len;
};

__device__ __forceinline__ bool wait_tc(unsigned long long* b, uint32_t parity, volatile int* abort) {
    if (c_force_wait_timeout) {
        *abort = 1;
        atomicOr(&g_device_error_tc, 2);
        return false;
    }
    return mbar_wait(b, parity, abort, &g_device_error_tc);
}
// Bounded wait that ignores the abort flag: the end-of-kernel drain of a thread's own
// MMAs (tensor memory may only be freed once nothing writes it any more).
__device__ __forceinline__ void drain_wait(unsigned long long* b, uint32_t parity = 0) {
    const uint32_t a = smem_u32(b);
    const long long t0 = clock64();
    while (true) {
        uint32_t ok;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
            : "=r"(ok)
            : "r"(a), "r"(parity)
            : "memory");
        if (ok) return;
        if (clock64() - t0 > WAIT_CYCLES) {
            atomicOr(&g_device_error_tc, 4);
            return;
        }
    }
}

template <typename T>
__device__ __forceinline__ uint4 nan_pack();
template <>
__device__ __forceinline__ uint4 nan_pack<__half>() { return make_uint4(0x7E007E00u, 0x7E007E00u, 0x7E007E00u, 0x7E007E00u); }
template <>
__device__ __forceinline__ uint4 nan_pack<__nv_bfloat16>() { return make_uint4(0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u); }

// ---------------------------------------------------------------------------
template <typename T, typename TW, bool TRANS>
__global__ void __launch_bounds__(NT, 1) wkv7_fwd_tc_kernel(const TcArgs p, const __grid_constant__ InMaps maps) {
    constexpr int ROWS = TRANS ? 128 : 64;
    using R = RawT<T, TW>;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    Smem<ROWS>& sm = *reinterpret_cast<Smem<ROWS>*>(smem_raw);
    // [2 groups][R::BYTES], 1024-byte aligned for the swizzled TMA boxes
    const uint32_t sbase = smem_u32(smem_raw);
    unsigned char* rawbuf = smem_raw + (((sbase + (uint32_t)sizeof(Smem<ROWS>) + 1023u) & ~1023u) - sbase);

    const int tid = threadIdx.x, warp = tid >> 5;
    const int nsl = TRANS ? p.nseg - 1 : p.nseg;  // segments in this launch
    const int bh = blockIdx.x / nsl, seg = blockIdx.x % nsl, H = p.H;
    const int bi = bh / H, hi = bh % H;
    const int t_begin = seg * p.seg_len;
    const int nloc = min(p.T, t_begin + p.seg_len) - t_begin;  // steps of this segment
    const size_t tstride = (size_t)H * N;
    const size_t base = (((size_t)bi * p.T + t_begin) * H + hi) * N;
    const int nchunks = (nloc + L - 1) / L;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                         smem_u32(&sm.tmem_base))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 32) {
        for (int i = 0; i < NSTAGE; i++) {
            mbar_init(&sm.full[i], 129);  // 128 prep threads + the commit of the X product
            mbar_init(&sm.empty[i], 128);
        }
        mbar_init(&sm.mma1, 4);  // one commit per state warp
        mbar_init(&sm.mma2, 1);
        mbar_init(&sm.drain[0], 1);
        mbar_init(&sm.drain[1], 1);
        mbar_init(&sm.drain[2], 4);
        mbar_init(&sm.ld_full[0], 1);
        mbar_init(&sm.ld_full[1], 1);
        sm.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if constexpr (TRANS) {  // rows 64..127 of V^T (the M part has no input) stay zero
        for (int s = 0; s < NSTAGE; s++)
            for (int i = tid; i < 8 * SBO_K16 / 16; i += NT)
                reinterpret_cast<uint4*>(sm.st[s].VT + 8 * SBO_K16)[i] = make_uint4(0, 0, 0, 0);
        proxy_fence();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;

    if (warp >= 4) {
        // ===================== prep groups =====================
        const int g_ = (warp - 4) >> 2;
        const int pt = tid - 128 - 128 * g_, pw = pt >> 5, lane = pt & 31, g = lane >> 2, tg = lane & 3;
        const int BAR = BAR_PREP0 + g_;
        PrepScratch& ps = sm.ps[g_];
        unsigned char* raw = rawbuf + (size_t)g_ * R::BYTES;

        // inputs of chunk c: one TMA box per array, issued by lane 0 of the group's warp 3
        // (which has no share of the forward substitution that follows the issue); the
        // group's k-th chunk (c = g_ + 2k) completes phase k of ld_full[g_]
        const int t_abs = t_begin;
        constexpr int ISSUER = 96;
        if (pt == ISSUER) {
#pragma unroll
            for (int i = 0; i < 6; i++)
                asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.m[i])) : "memory");
        }
        auto issue = [&](int c) {
            if (pt == ISSUER) {
                proxy_fence();  // the group's generic reads of the staging precede the TMA writes
                expect_tx(&sm.ld_full[g_], R::BYTES);
                const int tt = t_abs + c * L;
#pragma unroll
                for (int i = 0; i < 5; i++) wst::load_box<T>(raw + i * R::ARR, &maps.m[i], tt, hi, bi, &sm.ld_full[g_]);
                wst::load_box<TW>(raw + 5 * R::ARR, &maps.m[5], tt, hi, bi, &sm.ld_full[g_]);
            }
        };
        int n_issued = 0, n_used = 0;
        if (g_ < nchunks) issue(g_), n_issued++;
        for (int c = g_; c < nchunks; c += 2) {
            bool bad = !wait_tc(&sm.ld_full[g_], n_used & 1, &sm.abort);
            if (!bad) n_used++;
            const int si = c % NSTAGE;
            Stage<ROWS>& stg = sm.st[si];
            if (!bad && c >= NSTAGE) bad = !wait_tc(&sm.empty[si], ((c / NSTAGE) + 1) & 1, &sm.abort);
            if (group_sync_or(BAR, bad)) break;

            // ---- P1: cumulative log2 decay, decayed factors, operands ----
            const int t = lane & 15, cg = 2 * pw + (lane >> 4), j0 = 8 * cg;
            const bool tok = t < nloc - c * L;
            float wv[8], cs[8], cp[8], cl[8];
            wst::box8<TW>(raw + 5 * R::ARR, t, j0, wv);
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
                const float u = __shfl_up_sync(0xffffffffu, cs[q], 1, 16);
                cp[q] = t ? u : 0.f;
                cl[q] = __shfl_sync(0xffffffffu, cs[q], 15, 16);
                ext |= cl[q] < -115.f;  // cumulative decay below e^-80
            }
            float xr[8], xk[8], xv[8], xa[8], xb[8], o1[8], o2[8];
            wst::box8<T>(raw + 0 * R::ARR, t, j0, xr);
            wst::box8<T>(raw + 1 * R::ARR, t, j0, xk);
            wst::box8<T>(raw + 2 * R::ARR, t, j0, xv);
            wst::box8<T>(raw + 3 * R::ARR, t, j0, xa);
            wst::box8<T>(raw + 4 * R::ARR, t, j0, xb);
            float ec[8], ei[8], eL[8];
#pragma unroll
            for (int q = 0; q < 8; q++) {
                ec[q] = ex2(cs[q]);
                ei[q] = ex2(-cs[q]);
                eL[q] = ex2(cl[q] - cs[q]);
            }
#pragma unroll
            for (int q = 0; q < 8; q++) o1[q] = tf32f(xa[q] * ex2(cp[q])), o2[q] = tf32f(xr[q] * ec[q]);
            sts8(&ps.At[t][j0], o1);
            sts8(&ps.Rt[t][j0], o2);
#pragma unroll
            for (int q = 0; q < 8; q++) o1[q] = tf32f(xb[q] * ei[q]), o2[q] = tf32f(xk[q] * ei[q]);
            sts8(&ps.Bh[t][j0], o1);
            sts8(&ps.Kh[t][j0], o2);
#pragma unroll
            for (int q = 0; q < 8; q++) {
                const int key = j0 + q;
                *reinterpret_cast<float*>(stg.BB + kmaj(key, t, SBO_K16)) = tf32f(xb[q] * eL[q]);
                *reinterpret_cast<float*>(stg.BX + kmaj(2 * L + key, t, SBO_K16)) = tf32f(xk[q] * eL[q]);
                *reinterpret_cast<float*>(stg.VT + kmaj(key, t, SBO_K16)) = tf32f(xv[q]);  // key index = value index
            }
            sts8(&ps.Cs[t + 1][j0], cs);
            if (t == 0) {
#pragma unroll
                for (int q = 0; q < 8; q++) ps.Cs[0][j0 + q] = 0.f;
            }
            if (t == 15) sts8(&stg.GL[j0], ec);
            const bool extreme = group_sync_or(BAR, ext);

            // ---- P2: intra-chunk matrices (the transition pass needs only Mab, Mak) ----
            if (!extreme && (!TRANS || pw < 2)) {
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
            } else if (extreme) {
                for (int e = pt; e < (TRANS ? 2 : 4) * L * L; e += 128) {
                    const int which = e / (L * L), tt = (e / L) % L, sidx = e % L;
                    const bool strict = which < 2;
                    float val = 0.f;
                    if (strict ? (sidx < tt) : (sidx <= tt)) {
                        const int la = which < 2 ? 3 : 0, ra = (which & 1) ? 1 : 4;
                        const float* cl2 = (which < 2) ? ps.Cs[tt] : ps.Cs[tt + 1];
                        const float* cr2 = ps.Cs[sidx + 1];
                        for (int jj = 0; jj < N; jj++)
                            val = fmaf(wst::box1<T>(raw + la * R::ARR, tt, jj) * wst::box1<T>(raw + ra * R::ARR, sidx, jj),
                                        exp2f(cl2[jj] - cr2[jj]), val);
                    }
                    float(*Mo)[LDM] = which == 0 ? ps.Mab : which == 1 ? ps.Mak : which == 2 ? ps.Mrb : ps.Mrk;
                    Mo[tt][sidx] = which == 0 ? val : tf32f(val);
                }
            }
            group_sync(BAR);
            if (c + 2 < nchunks) issue(c + 2), n_issued++;  // raw staging is free from here on

            // ---- P4: forward substitution (I - Mab) X = [At | Mak]: Wu -> WB rows 0-15
            //      (threads 0-63, one key column each), Gu^T (threads 64-79) ----
            if (pt < N + L) {
                float x[L];
                const bool left = pt < N;
                const int col = left ? pt : pt - N;
#pragma unroll
                for (int tt = 0; tt < L; tt++) {  // Mab rows read as 16-byte vectors (4x fewer loads)
                    float accx = left ? ps.At[tt][col] : ps.Mak[tt][col];
#pragma unroll
                    for (int q = 0; q < (tt + 3) / 4; q++) {
                        const float4 m = *reinterpret_cast<const float4*>(&ps.Mab[tt][4 * q]);
                        if (4 * q + 0 < tt) accx = fmaf(m.x, x[4 * q + 0], accx);
                        if (4 * q + 1 < tt) accx = fmaf(m.y, x[4 * q + 1], accx);
                        if (4 * q + 2 < tt) accx = fmaf(m.z, x[4 * q + 2], accx);
                        if (4 * q + 3 < tt) accx = fmaf(m.w, x[4 * q + 3], accx);
                    }
                    x[tt] = accx;
                }
                if (left) {
#pragma unroll
                    for (int tt = 0; tt < L; tt++) *reinterpret_cast<float*>(stg.WB + kmaj(tt, col, SBO_K64)) = tf32f(x[tt]);
                } else {
#pragma unroll
                    for (int tt = 0; tt < L; tt++) ps.GuT[tt][col] = tf32f(x[tt]);
                }
            }
            group_sync(BAR);

            // ---- P5: Wy = Rt + Mrb Wu (WB rows 16-31); Gu^T, Gy^T = Mrb Gu^T + Mrk (BX rows 0-31).
            //      The transition pass produces no y: only Gu^T is needed (Wy, Gy rows stay unused) ----
            if constexpr (TRANS) {
                if (pw == 1) {
#pragma unroll
                    for (int i = 0; i < (L * L) / 32; i++) {
                        const int q = lane + 32 * i, tp = q / L, ss = q % L;
                        *reinterpret_cast<float*>(stg.BX + kmaj(tp, ss, SBO_K16)) = ps.GuT[tp][ss];
                    }
                }
            } else {
                auto ldB = [&](const unsigned char* src, int kk, int nn) {
                    return fbits(*reinterpret_cast<const float*>(src + kmaj(kk, nn, SBO_K64)));
                };
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
                        mma8(wy[nt], a0, a1, a2, a3, ldB(stg.WB, k0 + tg, n0 + g), ldB(stg.WB, k0 + tg + 4, n0 + g));
                    }
                }
#pragma unroll
                for (int nt = 0; nt < 2; nt++) {
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int tt = L + g + (e >> 1) * 8, col = 16 * pw + 8 * nt + 2 * tg + (e & 1);
                        *reinterpret_cast<float*>(stg.WB + kmaj(tt, col, SBO_K64)) = tf32f(wy[nt][e]);
                    }
                }
                // Gy^T = Mrb Gu^T + Mrk: one 16x8 tile each for warps 2 and 3; Gu^T copied
                // into BX by warps 0 and 1 (half each), so the four warps finish together
                if (pw >= 2) {
                    const int nt = pw - 2, n0 = 8 * nt + 2 * tg;
                    float gy[4] = {ps.Mrk[g][n0], ps.Mrk[g][n0 + 1], ps.Mrk[g + 8][n0], ps.Mrk[g + 8][n0 + 1]};
#pragma unroll
                    for (int ks = 0; ks < 2; ks++) {
                        const int k0 = 8 * ks;
                        const uint32_t a0 = fbits(ps.Mrb[g][k0 + tg]), a1 = fbits(ps.Mrb[g + 8][k0 + tg]);
                        const uint32_t a2 = fbits(ps.Mrb[g][k0 + tg + 4]), a3 = fbits(ps.Mrb[g + 8][k0 + tg + 4]);
                        mma8(gy, a0, a1, a2, a3, fbits(ps.GuT[k0 + tg][8 * nt + g]), fbits(ps.GuT[k0 + tg + 4][8 * nt + g]));
                    }
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int tp = g + (e >> 1) * 8, ss = 8 * nt + 2 * tg + (e & 1);
                        *reinterpret_cast<float*>(stg.BX + kmaj(L + tp, ss, SBO_K16)) = tf32f(gy[e]);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < (L * L) / 64; i++) {
                        const int q = lane + 32 * (2 * i + pw), tp = q / L, ss = q % L;
                        *reinterpret_cast<float*>(stg.BX + kmaj(tp, ss, SBO_K16)) = ps.GuT[tp][ss];
                    }
                }
            }
            proxy_fence();  // make the operand stores visible to the tensor cores
            group_sync(BAR);
            if (pt == 0) {
                // X = V^T [Gu | Gy | Kb] into this stage's tensor-memory columns; its
                // completion is the 129th arrival on the stage's full barrier
                tc_fence_after();
                const uint32_t ix = idesc_tf32(ROWS, 96), aV = smem_u32(stg.VT), bX = smem_u32(stg.BX);
#pragma unroll
                for (int ks = 0; ks < 2; ks++)
                    umma(tmem + COL_X + 96 * si, umma_desc(aV + 2 * ks * KLBO, SBO_K16),
                         umma_desc(bX + 2 * ks * KLBO, SBO_K16), ix, ks);
                umma_commit(&sm.full[si]);
            }
            mbar_arrive(&sm.full[si]);
        }
        if (pt == 0) {
            // a load issued but never waited for (the loop was left early) must land before
            // the shared memory is released; then this thread's own MMAs, before the tensor
            // memory is freed
            if (n_issued > n_used) drain_wait(&sm.ld_full[g_], (n_issued - 1) & 1);
            umma_commit(&sm.drain[g_]);
            drain_wait(&sm.drain[g_]);
        }
    } else {
        // ===================== state warps =====================
        // M=64: row i of the state lives in lane 16*(i/16) + i%16 of warp i/16's 32-lane
        // slice (lanes 0-15 of each slice); M=128 (transition): row i in lane i.
        const int tw = warp, lane = tid & 31;
        const bool live = TRANS || lane < 16;
        const int row = TRANS ? 32 * tw + lane : 16 * tw + lane;
        const uint32_t lb = (uint32_t)(32 * tw) << 16;
        const uint32_t tS = tmem + lb + COL_S;
        {
            float S[N];
            const float* src = nullptr;
            if (TRANS) {
                if (row < N && seg == 0 && p.s0) src = p.s0 + ((size_t)bh * N + row) * N;
            } else if (live) {
                if (seg == 0) {
                    if (p.s0) src = p.s0 + ((size_t)bh * N + row) * N;
                } else {
                    src = p.seg_s0 + (((size_t)bh * p.nseg + seg) * N + row) * N;
                }
            }
#pragma unroll
            for (int j = 0; j < N; j++) S[j] = src ? src[j] : ((TRANS && row - N == j) ? 1.f : 0.f);
#pragma unroll
            for (int j = 0; j < N; j += 16) tmem_st16(tS + j, &S[j]);
            tmem_wait_st();
        }
        bool bad_prev = false;  // a wait of the previous chunk gave up (voted on below)
        for (int c = 0; c < nchunks; c++) {
            const int si = c % NSTAGE;
            Stage<ROWS>& stg = sm.st[si];
            const uint32_t tX = tmem + lb + COL_X + 96 * si;
            const bool bad = bad_prev || !wait_tc(&sm.full[si], (c / NSTAGE) & 1, &sm.abort);
            if (group_sync_or(BAR_STATE, bad)) break;
            tc_fence_after();
            if (lane == 0) {
                // D1_w = S0[:, keys 16w..16w+15] [Wu; Wy][:, same keys]^T: 2 of the 8 K-steps
                const uint32_t i1 = idesc_tf32(ROWS, 32), bW = smem_u32(stg.WB);
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const int ks = 2 * tw + j;
                    umma_ts(tmem + COL_D1 + 32 * tw, tmem + COL_S + 8 * ks, umma_desc(bW + 2 * ks * KLBO, SBO_K64), i1, j);
                }
                umma_commit(&sm.mma1);
            }
            __syncwarp();
            const bool bad2 = !wait_tc(&sm.mma1, c & 1, &sm.abort);
            tc_fence_after();
            float u[L];
            {
                float p0[16], p1[16], p2[16], p3[16], px[16];
                tmem_ld16(tmem + lb + COL_D1, p0);
                tmem_ld16(tmem + lb + COL_D1 + 32, p1);
                tmem_ld16(tmem + lb + COL_D1 + 64, p2);
                tmem_ld16(tmem + lb + COL_D1 + 96, p3);
                tmem_ld16(tX, px);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < L; i++) u[i] = ((p0[i] + p1[i]) + (p2[i] + p3[i])) + px[i];
                float ut[L];
#pragma unroll
                for (int i = 0; i < L; i++) ut[i] = tf32f(u[i]);
                tmem_st16(tmem + lb + COL_U, ut);
            }
            if constexpr (!TRANS) {  // y rows of this chunk (D1's Wy parts + X's Yi part) into Yb
                float p0[16], p1[16], p2[16], p3[16], px[16];
                tmem_ld16(tmem + lb + COL_D1 + L, p0);
                tmem_ld16(tmem + lb + COL_D1 + 32 + L, p1);
                tmem_ld16(tmem + lb + COL_D1 + 64 + L, p2);
                tmem_ld16(tmem + lb + COL_D1 + 96 + L, p3);
                tmem_ld16(tX + L, px);
                tmem_wait_ld();
                if (live) {
#pragma unroll
                    for (int i = 0; i < L; i++) sm.Yb[i][row] = ((p0[i] + p1[i]) + (p2[i] + p3[i])) + px[i];
                }
            }
            // state * chunk decay + V^T Kb, two 32-column halves
#pragma unroll
            for (int j = 0; j < N; j += 32) {
                float s0v[16], s1v[16], x0[16], x1[16];
                tmem_ld16(tS + j, s0v);
                tmem_ld16(tS + j + 16, s1v);
                tmem_ld16(tX + 2 * L + j, x0);
                tmem_ld16(tX + 2 * L + j + 16, x1);
                tmem_wait_ld();
#pragma unroll
                for (int q = 0; q < 16; q += 4) {
                    const float4 g0 = *reinterpret_cast<const float4*>(&stg.GL[j + q]);
                    const float4 g1 = *reinterpret_cast<const float4*>(&stg.GL[j + 16 + q]);
                    s0v[q] = fmaf(s0v[q], g0.x, x0[q]), s0v[q + 1] = fmaf(s0v[q + 1], g0.y, x0[q + 1]);
                    s0v[q + 2] = fmaf(s0v[q + 2], g0.z, x0[q + 2]), s0v[q + 3] = fmaf(s0v[q + 3], g0.w, x0[q + 3]);
                    s1v[q] = fmaf(s1v[q], g1.x, x1[q]), s1v[q + 1] = fmaf(s1v[q + 1], g1.y, x1[q + 1]);
                    s1v[q + 2] = fmaf(s1v[q + 2], g1.z, x1[q + 2]), s1v[q + 3] = fmaf(s1v[q + 3], g1.w, x1[q + 3]);
                }
                tmem_st16(tS + j, s0v);
                tmem_st16(tS + j + 16, s1v);
            }
            tmem_wait_st();
            tc_fence_before();
            if (group_sync_or(BAR_STATE, bad2)) break;  // (also: Yb complete)
            tc_fence_after();
            if (tid == 0) {  // S_L += U^T Bb, A = U read from tensor memory
                const uint32_t i2 = idesc_tf32(ROWS, 64), bB = smem_u32(stg.BB);
#pragma unroll
                for (int ks = 0; ks < 2; ks++)
                    umma_ts(tmem + COL_S, tmem + COL_U + 8 * ks, umma_desc(bB + 2 * ks * KLBO, SBO_K16), i2, 1);
                umma_commit(&sm.mma2);
            }
            __syncwarp();
            if constexpr (!TRANS) {
                if (live && p.sa) {
#pragma unroll
                    for (int tt = 0; tt < L; tt++)
                        if (c * L + tt < nloc) p.sa[base + (size_t)(c * L + tt) * tstride + row] = u[tt];
                }
                {  // y rows of this chunk: values c4..c4+3 and 32+c4..35+c4 per thread (8 lanes
                   // read 128 contiguous bytes of Yb: conflict-free), two 8-byte stores
                    const int rr = tid >> 3, c4 = (tid & 7) * 4, t = c * L + rr;
                    if (t < nloc) {
#pragma unroll
                        for (int hh = 0; hh < 2; hh++) {
                            const float4 f = *reinterpret_cast<const float4*>(&sm.Yb[rr][32 * hh + c4]);
                            uint2 pk;
                            T* pe = reinterpret_cast<T*>(&pk);
                            pe[0] = from_f32<T>(f.x), pe[1] = from_f32<T>(f.y), pe[2] = from_f32<T>(f.z), pe[3] = from_f32<T>(f.w);
                            *reinterpret_cast<uint2*>((T*)p.y + base + (size_t)t * tstride + 32 * hh + c4) = pk;
                        }
                    }
                }
            }
            const bool bad3 = !wait_tc(&sm.mma2, c & 1, &sm.abort);
            tc_fence_after();
            if constexpr (!TRANS) {
                const int tend = t_begin + (c + 1) * L;  // global step index of the chunk end
                if (p.ckpt && tend <= p.T && tend % p.ckpt_len == 0) {
                    float S[N];
#pragma unroll
                    for (int j = 0; j < N; j += 16) tmem_ld16(tS + j, &S[j]);
                    tmem_wait_ld();
                    if (live) {
                        const int nck = p.T / p.ckpt_len;
                        float* q = p.ckpt + (((size_t)bh * nck + tend / p.ckpt_len - 1) * N + row) * N;
#pragma unroll
                        for (int j = 0; j < N; j += 4) *reinterpret_cast<float4*>(q + j) = make_float4(S[j], S[j + 1], S[j + 2], S[j + 3]);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&sm.empty[si]);
            bad_prev = bad3;  // the next chunk's first barrier decides for the whole group
        }
        if (group_sync_or(BAR_STATE, bad_prev)) sm.abort = 1;
        float* dst = nullptr;
        if (TRANS)
            dst = p.trans + (((size_t)bh * (p.nseg - 1) + seg) * ROWS + row) * N;
        else if (seg == p.nseg - 1 && p.sT && live)
            dst = p.sT + ((size_t)bh * N + row) * N;
        if (!group_sync_or(BAR_STATE, sm.abort != 0)) {
            tc_fence_after();
            float S[N];
#pragma unroll
            for (int j = 0; j < N; j += 16) tmem_ld16(tS + j, &S[j]);
            tmem_wait_ld();
            if (dst) {
#pragma unroll
                for (int j = 0; j < N; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(S[j], S[j + 1], S[j + 2], S[j + 3]);
            }
        }
        if (lane == 0) {  // wait for this warp's own MMAs before the tensor memory is freed
            umma_commit(&sm.drain[2]);
            drain_wait(&sm.drain[2]);
        }
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (sm.abort) {  // a wait gave up: no output of this CTA may look valid
        const float fnan = __int_as_float(0x7fc00000);
        if (TRANS) {
            float* o = p.trans + ((size_t)bh * (p.nseg - 1) + seg) * ROWS * N;
            for (int i = tid; i < ROWS * N; i += NT) o[i] = fnan;
        } else {
            for (int i = tid; i < nloc * 8; i += NT)
                *reinterpret_cast<uint4*>((T*)p.y + base + (size_t)(i >> 3) * tstride + (i & 7) * 8) = nan_pack<T>();
            if (p.sa)
                for (int i = tid; i < nloc * N; i += NT) p.sa[base + (size_t)(i >> 6) * tstride + (i & 63)] = fnan;
            if (p.sT && seg == p.nseg - 1)
                for (int i = tid; i < N * N; i += NT) p.sT[(size_t)bh * N * N + i] = fnan;
            if (p.ckpt) {
                const int nck = p.T / p.ckpt_len;
                for (int ck_i = 0; ck_i < nck; ck_i++) {
                    const int tend = (ck_i + 1) * p.ckpt_len;
                    if (tend <= t_begin || tend > t_begin + nloc) continue;
                    float* q = p.ckpt + ((size_t)bh * nck + ck_i) * N * N;
                    for (int i = tid; i < N * N; i += NT) q[i] = fnan;
                }
            }
        }
    }
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
}

// Composes the segments' affine maps: S_1 = C_0 (segment 0 started from the sequence's
// own initial state), S_{s+1} = S_s M_s + C_s.  Rows of the state are independent, so
// each CTA owns 8 rows of one (b, h); fp32 FMA.  The next segment's M (16 KB) and C rows
// are prefetched with cp.async while the current step computes, so a step costs its
// arithmetic, not a global-memory round trip.
__global__ void __launch_bounds__(256) wkv7_seg_scan_kernel(const float* __restrict__ trans,
                                                            float* __restrict__ seg_s0, int nseg) {
    __shared__ __align__(16) float M[2][N][N];
    __shared__ __align__(16) float Cr[2][8][N];
    __shared__ float S[8][N];
    const int bh = blockIdx.x, r0 = 8 * blockIdx.y, tid = threadIdx.x;
    const int i = tid >> 5, c0 = tid & 31, c1 = c0 + 32;
    const size_t cm = (size_t)ROWS_CM * N;
    const float* CM0 = trans + (size_t)bh * (nseg - 1) * cm;
    auto fetch = [&](int s, int buf) {  // M rows (16 KB) and this CTA's 8 C rows of segment s
        const float* CM = CM0 + (size_t)s * cm;
        for (int q = tid; q < N * N / 4; q += 256) cp_async16(&M[buf][0][0] + 4 * q, CM + (size_t)N * N + 4 * q, true);
        if (tid < 8 * N / 4) cp_async16(&Cr[buf][0][0] + 4 * tid, CM + (size_t)r0 * N + 4 * tid, true);
        cp_commit();
    };
    float s0v = CM0[(size_t)(r0 + i) * N + c0], s1v = CM0[(size_t)(r0 + i) * N + c1];
    if (nseg > 2) fetch(1, 1);
    float* out = seg_s0 + (((size_t)bh * nseg + 1) * N + r0 + i) * N;
    out[c0] = s0v, out[c1] = s1v;
    S[i][c0] = s0v, S[i][c1] = s1v;
    for (int s = 1; s < nseg - 1; s++) {
        const int buf = s & 1;
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();  // M[buf], Cr[buf] and S are complete
        if (s + 1 < nseg - 1) fetch(s + 1, buf ^ 1);
        float a0 = Cr[buf][i][c0], a1 = Cr[buf][i][c1];
#pragma unroll 16
        for (int j = 0; j < N; j++) {
            const float sj = S[i][j];
            a0 = fmaf(sj, M[buf][j][c0], a0);
            a1 = fmaf(sj, M[buf][j][c1], a1);
        }
        __syncthreads();  // every thread has read S
        S[i][c0] = a0, S[i][c1] = a1;
        out = seg_s0 + (((size_t)bh * nseg + s + 1) * N + r0 + i) * N;
        out[c0] = a0, out[c1] = a1;
    }
}

template <typename T, typename TW, bool TRANS>
size_t smem_bytes() {
    return sizeof(Smem<TRANS ? 128 : 64>) + 1024 /* alignment of the staging */ + 2 * (size_t)RawT<T, TW>::BYTES;
}

template <typename T, typename TW, bool TRANS>
int launch(const TcArgs& a, const InMaps& maps, int grid, cudaStream_t st) {
    auto kern = wkv7_fwd_tc_kernel<T, TW, TRANS>;
    const size_t smem = smem_bytes<T, TW, TRANS>();
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_cuda_error(e);
    kern<<<grid, NT, smem, st>>>(a, maps);
    return check_launch();
}

template <typename T, typename TW>
int make_in_maps(const WkvFwdArgs& p, InMaps& maps) {
    const void* src[5] = {p.r, p.k, p.v, p.a, p.b};
    for (int i = 0; i < 5; i++)
        if (wst::make_box_map<T>(&maps.m[i], src[i], p.B, p.T, p.H)) return RWKV_ERR_CUDA;
    if (wst::make_box_map<TW>(&maps.m[5], p.w, p.B, p.T, p.H)) return RWKV_ERR_CUDA;
    return RWKV_OK;
}

template <typename T, typename TW>
int run(const WkvFwdArgs& p, int nseg, float* ws, cudaStream_t st) {
    const int nch = (p.T + L - 1) / L;
    const int seg_chunks = (nch + nseg - 1) / nseg;
    nseg = (nch + seg_chunks - 1) / seg_chunks;  // no empty segment
    TcArgs a{p.r, p.w, p.k, p.v, p.a, p.b, p.s0, p.y, p.sT, p.ckpt, p.sa, nullptr, nullptr,
             p.T, p.H, p.ckpt_len, nseg, seg_chunks * L};
    const int units = p.B * p.H;
    alignas(64) InMaps maps;
    int rc = make_in_maps<T, TW>(p, maps);
    if (rc) return rc;
    if (nseg > 1) {
        a.trans = ws;
        a.seg_s0 = ws + (size_t)units * (nseg - 1) * ROWS_CM * N;
        rc = launch<T, TW, true>(a, maps, units * (nseg - 1), st);
        if (rc) return rc;
        wkv7_seg_scan_kernel<<<dim3(units, N / 8), 256, 0, st>>>(a.trans, a.seg_s0, nseg);
        rc = check_launch();
        if (rc) return rc;
    }
    return launch<T, TW, false>(a, maps, units * nseg, st);
}

}  // namespace tc

bool wkv7_tc_supported(int dtype) { return dtype == RWKV_F16 || dtype == RWKV_BF16; }

size_t wkv7_tc_ws_bytes(int B, int T, int H, int nseg) {
    if (nseg <= 1) return 0;
    const int nch = (T + ck::L - 1) / ck::L;
    const int seg_chunks = (nch + nseg - 1) / nseg;
    nseg = (nch + seg_chunks - 1) / seg_chunks;
    if (nseg <= 1) return 0;
    const size_t units = (size_t)B * H;
    return units * ((size_t)(nseg - 1) * tc::ROWS_CM * ck::N + (size_t)nseg * ck::N) * ck::N * sizeof(float);
}

int wkv7_fwd_tc(const WkvFwdArgs& p, int nseg, float* ws, cudaStream_t st) {
    switch (p.dtype) {
        case RWKV_F16:
            if (p.w_dtype == RWKV_F16) return tc::run<__half, __half>(p, nseg, ws, st);
            if (p.w_dtype == RWKV_F32) return tc::run<__half, float>(p, nseg, ws, st);
            return RWKV_ERR_DTYPE;
        case RWKV_BF16:
            if (p.w_dtype == RWKV_BF16) return tc::run<__nv_bfloat16, __nv_bfloat16>(p, nseg, ws, st);
            if (p.w_dtype == RWKV_F32) return tc::run<__nv_bfloat16, float>(p, nseg, ws, st);
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

int set_force_wait_timeout_tc(int on) {
    const int v = on ? 1 : 0;
    return set_cuda_error(cudaMemcpyToSymbol(c_force_wait_timeout, &v, sizeof(int)));
}

int set_device_error_tc(int value) {
    return set_cuda_error(cudaMemcpyToSymbol(g_device_error_tc, &value, sizeof(int)));
}

}  // namespace rwkv

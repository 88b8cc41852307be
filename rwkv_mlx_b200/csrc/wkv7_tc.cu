// WKV-7 forward with the state products on the 5th-generation tensor cores:
// tcgen05.mma (kind::tf32, M=64) with accumulators in tensor memory.  Same chunk
// algebra as wkv7_chunk.cu (L = 16):
//
//   D1 = [U | Y]^T = S0 [Wu; Wy]^T + [Ui; Yi]^T          (M=64 values, N=32, K=64)
//   D2 = S_L       = S0 diag(GL) + V^T Kb + U^T Bb        (M=64 values, N=64 keys, K=16+16)
//
// The fp32 state lives in tensor memory (D2) for the whole sequence and is itself the
// A operand of D1 (A read from tensor memory, B = [Wu; Wy] K-major in shared memory).
// Per chunk the 4 state warps preload the intra-chunk part [Ui; Yi]^T into D1, one
// thread issues the 8 K-steps of D1 as two independent accumulation chains, the warps
// scale D2 by the chunk decay and read U and Y back, then D2 takes the rank-32 update.
// Two groups of 4 "prep" warps compute the inputs-only chunk operands (decay factors,
// intra-chunk products on mma.sync, triangular solve) for alternating chunks, writing
// them straight into the UMMA operand layout; the hand-offs are mbarriers with bounded
// waits (a CTA that gives up sets the device error word and exits, it never traps).
//
// Supported for fp16 / bf16 activations (w in the activation dtype or fp32); fp32
// activations use the mma.sync kernel (their input staging does not fit next to this
// kernel's shared memory).
#include <cfloat>

#include "chunk_common.cuh"
#include "common.cuh"
#include "tc_common.cuh"
#include "wkv7.cuh"

namespace rwkv {

__device__ int g_device_error_tc;

namespace tc {
using namespace ck;
using namespace tcc;

constexpr int NT = 384;
constexpr int NSTAGE = 3;  // operand stages for 2 prep groups: one chunk of slack
constexpr int SBO_K64 = 16 * KLBO, SBO_K32 = 8 * KLBO, SBO_K16 = 4 * KLBO;
constexpr int SZ_WB = 4 * SBO_K64;  // 32 rows x K=64
constexpr int SZ_BK = 8 * SBO_K32;  // 64 rows x K=32
constexpr int SZ_VT = 8 * SBO_K16;  // 64 rows x K=16
constexpr int SZ_BY = 4 * SBO_K16;  // 32 rows x K=16

struct __align__(128) Stage {
    unsigned char WB[SZ_WB];  // B of D1: rows t' (0-15 Wu, 16-31 Wy), K = key
    unsigned char BY[SZ_BY];  // B of the intra-chunk part V^T [Gu | Gy]: rows t' (0-15 Gu^T, 16-31 Gy^T), K = s
    unsigned char BK[SZ_BK];  // B of D2: rows key, K = t' (0-15 Bb, 16-31 Kb)
    unsigned char VT[SZ_VT];  // A of D2 (V part): rows value, K = t
    float GL[N];              // decay of the whole chunk per key
};
struct __align__(16) PrepScratch {
    float At[L][LD4], Rt[L][LD4], Bh[L][LD4], Kh[L][LD4];
    float Mab[L][LDM], Mak[L][LDM], Mrb[L][LDM], Mrk[L][LDM];
    float GuT[L][LDM];  // (I - Mab)^-1 Mak
    float Cs[L + 1][N];  // cumulative log2 decay, Cs[0] = 0
};
struct __align__(128) Smem {
    Stage st[NSTAGE];  // chunk c uses stage c % NSTAGE
    unsigned char UTA[SZ_VT]; // A of D2 (U part): rows value, K = t
    float Yb[L][LD8];
    PrepScratch ps[2];
    unsigned long long full[NSTAGE], empty[NSTAGE], mma1, mma2;
    uint32_t tmem_base;
    int abort;
};

enum { BAR_STATE = 1, BAR_PREP0 = 2 };  // BAR_PREP0 + g for prep group g

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
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 128;" ::"r"(
                         smem_u32(&sm.tmem_base))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 32) {
        for (int i = 0; i < NSTAGE; i++) {
            mbar_init(&sm.full[i], 128);
            mbar_init(&sm.empty[i], 128);
        }
        mbar_init(&sm.mma1, 1);
        mbar_init(&sm.mma2, 1);
        sm.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
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

        if (g_ < nchunks) issue(g_);
        for (int c = g_; c < nchunks; c += 2) {
            asm volatile("cp.async.wait_all;" ::: "memory");
            bool bad = false;
            const int si = c % NSTAGE;
            Stage& stg = sm.st[si];
            if (c >= NSTAGE) bad = !mbar_wait(&sm.empty[si], ((c / NSTAGE) + 1) & 1, &sm.abort, &g_device_error_tc);
            if (group_sync_or(BAR, bad)) break;

            // ---- P1: cumulative log2 decay, decayed factors, operands ----
            const int t = lane & 15, cg = 2 * pw + (lane >> 4), j0 = 8 * cg;
            const bool tok = t < T_ - c * L;
            float wv[8], cs[8], cp[8], cl[8];
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
                const float u = __shfl_up_sync(0xffffffffu, cs[q], 1, 16);
                cp[q] = t ? u : 0.f;
                cl[q] = __shfl_sync(0xffffffffu, cs[q], 15, 16);
                ext |= cl[q] < -115.f;  // cumulative decay below e^-80
            }
            float xr[8], xk[8], xv[8], xa[8], xb[8], o1[8], o2[8];
            lds8<T>(raw + 0 * R::ARR + t * R::PITCH + j0 * sizeof(T), xr);
            lds8<T>(raw + 1 * R::ARR + t * R::PITCH + j0 * sizeof(T), xk);
            lds8<T>(raw + 2 * R::ARR + t * R::PITCH + j0 * sizeof(T), xv);
            lds8<T>(raw + 3 * R::ARR + t * R::PITCH + j0 * sizeof(T), xa);
            lds8<T>(raw + 4 * R::ARR + t * R::PITCH + j0 * sizeof(T), xb);
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
                *reinterpret_cast<float*>(stg.BK + kmaj(key, t, SBO_K32)) = tf32f(xb[q] * eL[q]);
                *reinterpret_cast<float*>(stg.BK + kmaj(key, L + t, SBO_K32)) = tf32f(xk[q] * eL[q]);
                const float vq = tf32f(xv[q]);
                o1[q] = vq;
                *reinterpret_cast<float*>(stg.VT + kmaj(key, t, SBO_K16)) = vq;  // key index = value index
            }
            sts8(&ps.Cs[t + 1][j0], cs);
            if (t == 0) {
#pragma unroll
                for (int q = 0; q < 8; q++) ps.Cs[0][j0 + q] = 0.f;
            }
            if (t == 15) sts8(&stg.GL[j0], ec);
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

            // ---- P4: forward substitution (I - Mab) X = [At | Mak]: Wu -> WB rows 0-15
            //      (threads 0-63, one key column each), Gu^T (threads 64-79) ----
            if (pt < N + L) {
                float x[L];
                const bool left = pt < N;
                const int col = left ? pt : pt - N;
#pragma unroll
                for (int tt = 0; tt < L; tt++) {
                    float accx = left ? ps.At[tt][col] : ps.Mak[tt][col];
#pragma unroll
                    for (int s2 = 0; s2 < tt; s2++) accx = fmaf(ps.Mab[tt][s2], x[s2], accx);
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

            // ---- P5: Wy = Rt + Mrb Wu (WB rows 16-31); Gu^T, Gy^T = Mrb Gu^T + Mrk (BY) ----
            {
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
                if (pw == 0) {
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
                            *reinterpret_cast<float*>(stg.BY + kmaj(L + tp, ss, SBO_K16)) = tf32f(gy[nt][e]);
                        }
                    }
                } else if (pw == 1) {
#pragma unroll
                    for (int i = 0; i < (L * L) / 32; i++) {
                        const int q = lane + 32 * i, tp = q / L, ss = q % L;
                        *reinterpret_cast<float*>(stg.BY + kmaj(tp, ss, SBO_K16)) = ps.GuT[tp][ss];
                    }
                }
            }
            proxy_fence();  // make the operand stores visible to the tensor cores
            mbar_arrive(&sm.full[si]);
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else {
        // ===================== state warps =====================
        // TMEM columns: [0,64) D2 = state, [64,96) D1a, [96,128) D1b (D1 = D1a + D1b).
        const int tw = warp, lane = tid & 31;
        const bool live = lane < 16;              // M=64 accumulators use lanes 0-15 of each subpartition
        const int row = 16 * tw + lane;            // state row (value index) held by this thread
        const uint32_t lane_base = (uint32_t)(32 * tw) << 16;
        const uint32_t tD2 = tmem + lane_base, tD1a = tD2 + 64, tD1b = tD2 + 96;
        {
            float S[N];
            const float* p = (s0 && live) ? s0 + ((size_t)bh * N + row) * N : nullptr;
#pragma unroll
            for (int j = 0; j < N; j++) S[j] = p ? p[j] : 0.f;
#pragma unroll
            for (int j = 0; j < N; j += 16) tmem_st16(tD2 + j, &S[j]);
            tmem_wait_st();
        }
        bool bad_prev = false;  // a wait of the previous chunk gave up (voted on below)
        for (int c = 0; c < nchunks; c++) {
            const int s = c % NSTAGE;
            Stage& stg = sm.st[s];
            const bool bad = bad_prev || !mbar_wait(&sm.full[s], (c / NSTAGE) & 1, &sm.abort, &g_device_error_tc);
            if (group_sync_or(BAR_STATE, bad)) break;
            tc_fence_after();
            if (tid == 0) {
                // D1a = V^T [Gu | Gy] (intra-chunk part), then + S0 [Wu; Wy]^T over two chains
                const uint32_t i1 = idesc_tf32(64, 32), bW = smem_u32(stg.WB), aV = smem_u32(stg.VT),
                               bY = smem_u32(stg.BY);
#pragma unroll
                for (int ks = 0; ks < 2; ks++)
                    umma(tmem + 64, umma_desc(aV + 2 * ks * KLBO, SBO_K16), umma_desc(bY + 2 * ks * KLBO, SBO_K16), i1, ks);
#pragma unroll
                for (int ks = 0; ks < 8; ks++)
                    umma_ts((ks & 1) ? tmem + 96 : tmem + 64, tmem + 8 * ks, umma_desc(bW + 2 * ks * KLBO, SBO_K64), i1,
                            (ks & 1) ? (ks > 1) : 1);
                umma_commit(&sm.mma1);
            }
            const bool bad2 = !mbar_wait(&sm.mma1, c & 1, &sm.abort, &g_device_error_tc);
            tc_fence_after();
            float S[N], u[L], yv[L], u2[L], y2[L];
#pragma unroll
            for (int j = 0; j < N; j += 16) tmem_ld16(tD2 + j, &S[j]);
            tmem_ld16(tD1a, u);
            tmem_ld16(tD1a + 16, yv);
            tmem_ld16(tD1b, u2);
            tmem_ld16(tD1b + 16, y2);
            tmem_wait_ld();
            // state * chunk decay -> D2
#pragma unroll
            for (int j = 0; j < N; j += 4) {
                const float4 gl = *reinterpret_cast<const float4*>(&stg.GL[j]);
                S[j] *= gl.x, S[j + 1] *= gl.y, S[j + 2] *= gl.z, S[j + 3] *= gl.w;
            }
#pragma unroll
            for (int j = 0; j < N; j += 16) tmem_st16(tD2 + j, &S[j]);
            tmem_wait_st();
            tc_fence_before();
            group_sync(BAR_STATE);
            tc_fence_after();
            if (tid == 0) {  // V^T Kb needs only the rescaled state: start it while U is staged
                const uint32_t i2 = idesc_tf32(64, 64), aV = smem_u32(stg.VT), bK = smem_u32(stg.BK);
#pragma unroll
                for (int ks = 0; ks < 2; ks++)
                    umma(tmem, umma_desc(aV + 2 * ks * KLBO, SBO_K16), umma_desc(bK + (4 + 2 * ks) * KLBO, SBO_K32), i2, 1);
            }
#pragma unroll
            for (int tt = 0; tt < L; tt++) u[tt] += u2[tt], yv[tt] += y2[tt];
            if (live) {
#pragma unroll
                for (int tt = 0; tt < L; tt += 4) st4(sm.UTA + kmaj(row, tt, SBO_K16), u[tt], u[tt + 1], u[tt + 2], u[tt + 3]);
#pragma unroll
                for (int tt = 0; tt < L; tt++) sm.Yb[tt][row] = yv[tt];
                if (sa_out) {
#pragma unroll
                    for (int tt = 0; tt < L; tt++)
                        if (c * L + tt < T_) sa_out[base + (size_t)(c * L + tt) * tstride + row] = u[tt];
                }
            }
            tmem_wait_st();
            proxy_fence();
            tc_fence_before();
            if (group_sync_or(BAR_STATE, bad2)) break;
            tc_fence_after();
            if (tid == 0) {
                const uint32_t i2 = idesc_tf32(64, 64);
                const uint32_t aU = smem_u32(sm.UTA), bK = smem_u32(stg.BK);
#pragma unroll
                for (int ks = 0; ks < 2; ks++)
                    umma(tmem, umma_desc(aU + 2 * ks * KLBO, SBO_K16), umma_desc(bK + 2 * ks * KLBO, SBO_K32), i2, 1);
                umma_commit(&sm.mma2);
            }
            {  // y rows of this chunk: 8 consecutive values per thread, one 16-byte store
                const int rr = tid >> 3, c8 = (tid & 7) * 8, t = c * L + rr;
                if (t < T_) {
                    const float4 f0 = *reinterpret_cast<const float4*>(&sm.Yb[rr][c8]);
                    const float4 f1 = *reinterpret_cast<const float4*>(&sm.Yb[rr][c8 + 4]);
                    uint4 pk;
                    T* pe = reinterpret_cast<T*>(&pk);
                    pe[0] = from_f32<T>(f0.x), pe[1] = from_f32<T>(f0.y), pe[2] = from_f32<T>(f0.z), pe[3] = from_f32<T>(f0.w);
                    pe[4] = from_f32<T>(f1.x), pe[5] = from_f32<T>(f1.y), pe[6] = from_f32<T>(f1.z), pe[7] = from_f32<T>(f1.w);
                    *reinterpret_cast<uint4*>(y + base + (size_t)t * tstride + c8) = pk;
                }
            }
            const bool bad3 = !mbar_wait(&sm.mma2, c & 1, &sm.abort, &g_device_error_tc);
            tc_fence_after();
            if (ckpt) {
                const int tend = (c + 1) * L;
                if (tend <= T_ && tend % ckpt_len == 0) {
#pragma unroll
                    for (int j = 0; j < N; j += 16) tmem_ld16(tD2 + j, &S[j]);
                    tmem_wait_ld();
                    if (live) {
                        float* p = ckpt + (((size_t)bh * nck + tend / ckpt_len - 1) * N + row) * N;
#pragma unroll
                        for (int j = 0; j < N; j += 4) *reinterpret_cast<float4*>(p + j) = make_float4(S[j], S[j + 1], S[j + 2], S[j + 3]);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&sm.empty[s]);
            bad_prev = bad3;  // the next chunk's first barrier decides for the whole group
        }
        if (group_sync_or(BAR_STATE, bad_prev)) sm.abort = 1;
        if (sT && !group_sync_or(BAR_STATE, sm.abort != 0)) {
            tc_fence_after();
            float S[N];
#pragma unroll
            for (int j = 0; j < N; j += 16) tmem_ld16(tD2 + j, &S[j]);
            tmem_wait_ld();
            if (live) {
                float* p = sT + ((size_t)bh * N + row) * N;
#pragma unroll
                for (int j = 0; j < N; j += 4) *reinterpret_cast<float4*>(p + j) = make_float4(S[j], S[j + 1], S[j + 2], S[j + 3]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 128;" ::"r"(tmem) : "memory");
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

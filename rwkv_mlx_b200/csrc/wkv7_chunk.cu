// WKV-7 forward, chunked on tensor cores (mma.sync m16n8k8, TF32 operands with
// round-to-nearest, fp32 accumulate; the 64x64 state stays fp32).
//
// Chunk algebra (per head, chunk of L = 16 steps, S0 the state entering the chunk,
// c_t = sum_{s<=t} -exp(w_s) the cumulative log decay inside the chunk):
//   At = a * e^{c_{t-1}}   Rt = r * e^{c_t}   Bh = b * e^{-c_t}   Kh = k * e^{-c_t}
//   Bb = b * e^{c_L - c_t} Kb = k * e^{c_L - c_t}
//   Mab = strict_tril(At Bh^T)  Mak = strict_tril(At Kh^T)
//   Mrb = tril(Rt Bh^T)         Mrk = tril(Rt Kh^T)
//   Wu = (I - Mab)^-1 At        Ui = (I - Mab)^-1 Mak V
//   Wy = Rt + Mrb Wu            Yi = Mrb Ui + Mrk V
//   U  = Wu S0^T + Ui  (rows: sa_t = S_{t-1} a_t)      Y = Wy S0^T + Yi  (rows: y_t)
//   S_L^T = diag(e^{c_L}) S0^T + Bb^T U + Kb^T V
// which is the unrolled form of S_t = S_{t-1} diag(decay_t) + sa_t b_t^T + v_t k_t^T,
// y_t = S_t r_t (reference: rwkv_mlx/kernels/wkv7_metal.py:53-91).  Everything
// above the U/Y line depends on the inputs only; the CTA's 4 "prep" warps compute
// it one chunk ahead while the 4 "state" warps run the two state products.
//
// If a chunk's cumulative decay falls below e^-80 (per-step decays far below what
// the model produces, decay >= 0.545), e^{-c_t} could overflow; that chunk's four
// intra matrices are then formed element-wise from exponent differences instead.
#include <cfloat>

#include "chunk_common.cuh"
#include "common.cuh"
#include "wkv7.cuh"

namespace rwkv {

__device__ int g_device_error;  // set by a kernel that gave up a bounded wait

namespace ck {
constexpr int NT = 256;

struct __align__(16) Stage {
    float Wu[L][LD4];
    float Wy[L][LD4];
    float Ui[L][LD8];
    float Yi[L][LD8];
    float Bb[L][LD8];
    float Kb[L][LD8];
    float V[L][LD8];
    float GL[N];
};

struct __align__(16) Smem {
    Stage st[2];
    float S[N][LD4];  // state entering the chunk, S[value][key], tf32-rounded
    float Ub[L][LD8];
    float Yb[L][LD8];
    float At[L][LD4], Rt[L][LD4], Bh[L][LD4], Kh[L][LD4];
    float Mab[L][LDM], Mak[L][LDM], Mrb[L][LDM], Mrk[L][LDM];
    float MakV[L][LD8];
    float Cs[L + 1][LD4];  // cumulative log decay, Cs[0] = 0, Cs[t+1] = c_t (rows padded: conflict-free stores)
    unsigned long long full[2], empty[2];
    int abort;
};

enum { BAR_PREP = 1, BAR_STATE = 2 };

template <typename T, typename TW>
__global__ void __launch_bounds__(NT, 1)
    wkv7_fwd_chunk_kernel(const T* __restrict__ r, const TW* __restrict__ w, const T* __restrict__ k,
                          const T* __restrict__ v, const T* __restrict__ a, const T* __restrict__ b,
                          const float* __restrict__ s0, T* __restrict__ y, float* __restrict__ sT,
                          float* __restrict__ ckpt, float* __restrict__ sa_out, int T_, int H,
                          int ckpt_len) {
    using R = Raw<T, TW>;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
    unsigned char* rawbuf = smem_raw + ((sizeof(Smem) + 127) / 128) * 128;  // [2][R::BYTES]

    const int tid = threadIdx.x;
    const int bh = blockIdx.x, bi = bh / H, hi = bh % H;
    const size_t tstride = (size_t)H * N;
    const size_t base = ((size_t)bi * T_ * H + hi) * N;
    const int nchunks = (T_ + L - 1) / L;
    const int nck = ckpt ? T_ / ckpt_len : 0;

    if (tid == 0) {
        mbar_init(&sm.full[0], 128);
        mbar_init(&sm.full[1], 128);
        mbar_init(&sm.empty[0], 128);
        mbar_init(&sm.empty[1], 128);
        sm.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (tid >= 128) {
        // ===================== prep warps =====================
        const int pt = tid - 128, pw = pt >> 5, lane = pt & 31, g = lane >> 2, tg = lane & 3;

        // each thread's 16-byte pieces of a chunk, fixed across chunks
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
            unsigned char* dst = rawbuf + (size_t)(c & 1) * R::BYTES;
            const int t0 = c * L;
#pragma unroll
            for (int i = 0; i < R::PER_THREAD; i++) {
                if (prow[i] < 0) continue;
                const bool ok = (t0 + prow[i]) < T_;
                const size_t step = (size_t)t0 * tstride;
                const char* src = ok ? psrc[i] + step * (pdst[i] >= 5u * R::ARR ? sizeof(TW) : sizeof(T))
                                     : psrc[i];
                cp_async16(dst + pdst[i], src, ok);
            }
        };

        issue(0);
        cp_commit();
        for (int c = 0; c < nchunks; c++) {
            const int s = c & 1;
            Stage& stg = sm.st[s];
            if (c + 1 < nchunks) issue(c + 1);
            cp_commit();
            cp_wait1();
            bool bad = false;
            if (c >= 2) bad = !mbar_wait(&sm.empty[s], ((c >> 1) + 1) & 1, &sm.abort, &g_device_error);
            if (group_sync_or(BAR_PREP, bad)) break;

            // ---- P1: cumulative log2 decay and decayed factors ----
            // thread = (row t, 8 consecutive columns); the scan over t runs across the
            // 16 lanes that share a column group
            const unsigned char* raw = rawbuf + (size_t)s * R::BYTES;
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
            sts8(&sm.At[t][j0], o1);
            sts8(&sm.Rt[t][j0], o2);
#pragma unroll
            for (int q = 0; q < 8; q++) o1[q] = tf32f(xb[q] * ei[q]), o2[q] = tf32f(xk[q] * ei[q]);
            sts8(&sm.Bh[t][j0], o1);
            sts8(&sm.Kh[t][j0], o2);
#pragma unroll
            for (int q = 0; q < 8; q++) o1[q] = tf32f(xb[q] * eL[q]), o2[q] = tf32f(xk[q] * eL[q]);
            sts8(&stg.Bb[t][j0], o1);
            sts8(&stg.Kb[t][j0], o2);
#pragma unroll
            for (int q = 0; q < 8; q++) o1[q] = tf32f(xv[q]);
            sts8(&stg.V[t][j0], o1);
            sts8(&sm.Cs[t + 1][j0], cs);  // log2 units, used by the element-wise path
            if (t == 0) {
#pragma unroll
                for (int q = 0; q < 8; q++) sm.Cs[0][j0 + q] = 0.f;
            }
            if (t == 15) sts8(&stg.GL[j0], ec);
            const bool extreme = group_sync_or(BAR_PREP, ext);

            // ---- P2: intra-chunk matrices ----
            if (!extreme) {
                const float(*Am)[LD4] = (pw >> 1) ? sm.Rt : sm.At;
                const float(*Bm)[LD4] = (pw & 1) ? sm.Kh : sm.Bh;
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
                float(*Mo)[LDM] = pw == 0 ? sm.Mab : pw == 1 ? sm.Mak : pw == 2 ? sm.Mrb : sm.Mrk;
                const bool strict = pw < 2;
#pragma unroll
                for (int nt = 0; nt < 2; nt++) {
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int t = g + (e >> 1) * 8, sidx = 8 * nt + 2 * tg + (e & 1);
                        const bool keep = strict ? (sidx < t) : (sidx <= t);
                        const float val = keep ? acc2[nt][e] : 0.f;
                        Mo[t][sidx] = (pw == 0) ? val : tf32f(val);
                    }
                }
            } else {
                // element-wise from exponent differences (all exponents <= 0)
                for (int e = pt; e < 4 * L * L; e += 128) {
                    const int which = e / (L * L), tt = (e / L) % L, sidx = e % L;
                    const bool strict = which < 2;
                    float val = 0.f;
                    if (strict ? (sidx < tt) : (sidx <= tt)) {
                        const T* lhs = reinterpret_cast<const T*>(raw + (which < 2 ? 3 : 0) * R::ARR + tt * R::PITCH);
                        const T* rhs = reinterpret_cast<const T*>(raw + ((which & 1) ? 1 : 4) * R::ARR + sidx * R::PITCH);
                        const float* cl2 = (which < 2) ? sm.Cs[tt] : sm.Cs[tt + 1];
                        const float* cr2 = sm.Cs[sidx + 1];
                        for (int jj = 0; jj < N; jj++)
                            val = fmaf(to_f32(lhs[jj]) * to_f32(rhs[jj]), exp2f(cl2[jj] - cr2[jj]), val);
                    }
                    float(*Mo)[LDM] = which == 0 ? sm.Mab : which == 1 ? sm.Mak : which == 2 ? sm.Mrb : sm.Mrk;
                    Mo[tt][sidx] = which == 0 ? val : tf32f(val);
                }
            }
            group_sync(BAR_PREP);

            // ---- P3: MakV = Mak V ----
            {
                float acc3[2][4] = {};
#pragma unroll
                for (int ks = 0; ks < 2; ks++) {
                    const int k0 = 8 * ks;
                    const uint32_t a0 = fbits(sm.Mak[g][k0 + tg]), a1 = fbits(sm.Mak[g + 8][k0 + tg]);
                    const uint32_t a2 = fbits(sm.Mak[g][k0 + tg + 4]), a3 = fbits(sm.Mak[g + 8][k0 + tg + 4]);
#pragma unroll
                    for (int nt = 0; nt < 2; nt++) {
                        const int n0 = 16 * pw + 8 * nt;
                        mma8(acc3[nt], a0, a1, a2, a3, fbits(stg.V[k0 + tg][n0 + g]), fbits(stg.V[k0 + tg + 4][n0 + g]));
                    }
                }
#pragma unroll
                for (int nt = 0; nt < 2; nt++) {
                    const int n0 = 16 * pw + 8 * nt + 2 * tg;
                    *reinterpret_cast<float2*>(&sm.MakV[g][n0]) = make_float2(acc3[nt][0], acc3[nt][1]);
                    *reinterpret_cast<float2*>(&sm.MakV[g + 8][n0]) = make_float2(acc3[nt][2], acc3[nt][3]);
                }
            }
            group_sync(BAR_PREP);

            // ---- P4: forward substitution  X = (I - Mab)^-1 [At | MakV] ----
            {
                float x[L];
                const bool left = pt < 64;
                const int col = left ? pt : pt - 64;
#pragma unroll
                for (int t = 0; t < L; t++) {
                    float accx = left ? sm.At[t][col] : sm.MakV[t][col];
#pragma unroll
                    for (int s2 = 0; s2 < t; s2++) accx = fmaf(sm.Mab[t][s2], x[s2], accx);
                    x[t] = accx;
                }
                if (left) {
#pragma unroll
                    for (int t = 0; t < L; t++) stg.Wu[t][col] = tf32f(x[t]);
                } else {
#pragma unroll
                    for (int t = 0; t < L; t++) stg.Ui[t][col] = x[t];
                }
            }
            group_sync(BAR_PREP);

            // ---- P5: Wy = Rt + Mrb Wu ;  Yi = Mrb Ui + Mrk V ----
            {
                float wy[2][4], yi[2][4] = {};
#pragma unroll
                for (int nt = 0; nt < 2; nt++) {
                    const int n0 = 16 * pw + 8 * nt + 2 * tg;
                    wy[nt][0] = sm.Rt[g][n0], wy[nt][1] = sm.Rt[g][n0 + 1];
                    wy[nt][2] = sm.Rt[g + 8][n0], wy[nt][3] = sm.Rt[g + 8][n0 + 1];
                }
#pragma unroll
                for (int ks = 0; ks < 2; ks++) {
                    const int k0 = 8 * ks;
                    const uint32_t a0 = fbits(sm.Mrb[g][k0 + tg]), a1 = fbits(sm.Mrb[g + 8][k0 + tg]);
                    const uint32_t a2 = fbits(sm.Mrb[g][k0 + tg + 4]), a3 = fbits(sm.Mrb[g + 8][k0 + tg + 4]);
#pragma unroll
                    for (int nt = 0; nt < 2; nt++) {
                        const int n0 = 16 * pw + 8 * nt;
                        mma8(wy[nt], a0, a1, a2, a3, fbits(stg.Wu[k0 + tg][n0 + g]), fbits(stg.Wu[k0 + tg + 4][n0 + g]));
                        mma8(yi[nt], a0, a1, a2, a3, tf32(stg.Ui[k0 + tg][n0 + g]), tf32(stg.Ui[k0 + tg + 4][n0 + g]));
                    }
                    const uint32_t c0 = fbits(sm.Mrk[g][k0 + tg]), c1 = fbits(sm.Mrk[g + 8][k0 + tg]);
                    const uint32_t c2 = fbits(sm.Mrk[g][k0 + tg + 4]), c3 = fbits(sm.Mrk[g + 8][k0 + tg + 4]);
#pragma unroll
                    for (int nt = 0; nt < 2; nt++) {
                        const int n0 = 16 * pw + 8 * nt;
                        mma8(yi[nt], c0, c1, c2, c3, fbits(stg.V[k0 + tg][n0 + g]), fbits(stg.V[k0 + tg + 4][n0 + g]));
                    }
                }
#pragma unroll
                for (int nt = 0; nt < 2; nt++) {
                    const int n0 = 16 * pw + 8 * nt + 2 * tg;
                    stg.Wy[g][n0] = tf32f(wy[nt][0]);
                    stg.Wy[g][n0 + 1] = tf32f(wy[nt][1]);
                    stg.Wy[g + 8][n0] = tf32f(wy[nt][2]);
                    stg.Wy[g + 8][n0 + 1] = tf32f(wy[nt][3]);
                    *reinterpret_cast<float2*>(&stg.Yi[g][n0]) = make_float2(yi[nt][0], yi[nt][1]);
                    *reinterpret_cast<float2*>(&stg.Yi[g + 8][n0]) = make_float2(yi[nt][2], yi[nt][3]);
                }
            }
            mbar_arrive(&sm.full[s]);
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else {
        // ===================== state warps =====================
        const int sw = tid >> 5, lane = tid & 31, g = lane >> 2, tg = lane & 3;
        // persistent fp32 state: C fragments of S^T, keys 16sw..16sw+15 (rows) x 64 values
        float st[8][4];
        {
            const float* p = s0 ? s0 + (size_t)bh * N * N : nullptr;
#pragma unroll
            for (int nt = 0; nt < 8; nt++) {
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int key = 16 * sw + g + (e >> 1) * 8, val = 8 * nt + 2 * tg + (e & 1);
                    st[nt][e] = p ? p[(size_t)val * N + key] : 0.f;
                    sm.S[val][key] = tf32f(st[nt][e]);
                }
            }
        }
        group_sync(BAR_STATE);
        for (int c = 0; c < nchunks; c++) {
            const int s = c & 1;
            Stage& stg = sm.st[s];
            const bool bad = !mbar_wait(&sm.full[s], (c >> 1) & 1, &sm.abort, &g_device_error);
            if (group_sync_or(BAR_STATE, bad)) break;

            // ---- S1: [U; Y] = [Wu; Wy] S0^T + [Ui; Yi] ----
            {
                const int mt = sw >> 1, nb = 32 * (sw & 1);
                const float(*Am)[LD4] = mt ? stg.Wy : stg.Wu;
                const float(*Cm)[LD8] = mt ? stg.Yi : stg.Ui;
                float acc[4][4];
#pragma unroll
                for (int nt = 0; nt < 4; nt++) {
                    const int n0 = nb + 8 * nt + 2 * tg;
                    const float2 lo = *reinterpret_cast<const float2*>(&Cm[g][n0]);
                    const float2 hi2 = *reinterpret_cast<const float2*>(&Cm[g + 8][n0]);
                    acc[nt][0] = lo.x, acc[nt][1] = lo.y, acc[nt][2] = hi2.x, acc[nt][3] = hi2.y;
                }
#pragma unroll
                for (int ks = 0; ks < 8; ks++) {
                    const int k0 = 8 * ks;
                    const uint32_t a0 = fbits(Am[g][k0 + tg]), a1 = fbits(Am[g + 8][k0 + tg]);
                    const uint32_t a2 = fbits(Am[g][k0 + tg + 4]), a3 = fbits(Am[g + 8][k0 + tg + 4]);
#pragma unroll
                    for (int nt = 0; nt < 4; nt++) {
                        const int n0 = nb + 8 * nt;
                        mma8(acc[nt], a0, a1, a2, a3, fbits(sm.S[n0 + g][k0 + tg]), fbits(sm.S[n0 + g][k0 + tg + 4]));
                    }
                }
                float(*Out)[LD8] = mt ? sm.Yb : sm.Ub;
#pragma unroll
                for (int nt = 0; nt < 4; nt++) {
                    const int n0 = nb + 8 * nt + 2 * tg;
                    *reinterpret_cast<float2*>(&Out[g][n0]) = make_float2(acc[nt][0], acc[nt][1]);
                    *reinterpret_cast<float2*>(&Out[g + 8][n0]) = make_float2(acc[nt][2], acc[nt][3]);
                }
            }
            group_sync(BAR_STATE);

            // ---- S2: S_L^T = diag(GL) S0^T + Bb^T U + Kb^T V ----
            {
                const float gl0 = stg.GL[16 * sw + g], gl1 = stg.GL[16 * sw + g + 8];
#pragma unroll
                for (int nt = 0; nt < 8; nt++) {
                    st[nt][0] *= gl0, st[nt][1] *= gl0, st[nt][2] *= gl1, st[nt][3] *= gl1;
                }
#pragma unroll
                for (int ks = 0; ks < 4; ks++) {
                    const float(*Asrc)[LD8] = ks < 2 ? stg.Bb : stg.Kb;
                    const int t0 = 8 * (ks & 1), m0 = 16 * sw;
                    const uint32_t a0 = fbits(Asrc[t0 + tg][m0 + g]), a1 = fbits(Asrc[t0 + tg][m0 + g + 8]);
                    const uint32_t a2 = fbits(Asrc[t0 + tg + 4][m0 + g]), a3 = fbits(Asrc[t0 + tg + 4][m0 + g + 8]);
#pragma unroll
                    for (int nt = 0; nt < 8; nt++) {
                        const int n0 = 8 * nt;
                        uint32_t b0, b1;
                        if (ks < 2) {
                            b0 = tf32(sm.Ub[t0 + tg][n0 + g]), b1 = tf32(sm.Ub[t0 + tg + 4][n0 + g]);
                        } else {
                            b0 = fbits(stg.V[t0 + tg][n0 + g]), b1 = fbits(stg.V[t0 + tg + 4][n0 + g]);
                        }
                        mma8(st[nt], a0, a1, a2, a3, b0, b1);
                    }
                }
            }
            // new state -> shared (operand of the next chunk)
#pragma unroll
            for (int nt = 0; nt < 8; nt++) {
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int key = 16 * sw + g + (e >> 1) * 8, val = 8 * nt + 2 * tg + (e & 1);
                    sm.S[val][key] = tf32f(st[nt][e]);
                }
            }
            mbar_arrive(&sm.empty[s]);
            // outputs of this chunk: y (and sa) rows, coalesced
            {
                const int row = tid >> 3, c8 = (tid & 7) * 8, t = c * L + row;
                if (t < T_) {
                    const size_t off = base + (size_t)t * tstride + c8;
#pragma unroll
                    for (int q = 0; q < 8; q++) y[off + q] = from_f32<T>(sm.Yb[row][c8 + q]);
                    if (sa_out) {
#pragma unroll
                        for (int q = 0; q < 8; q++) sa_out[off + q] = sm.Ub[row][c8 + q];
                    }
                }
            }
            if (ckpt) {
                const int tend = (c + 1) * L;
                if (tend <= T_ && tend % ckpt_len == 0) {
                    float* p = ckpt + ((size_t)bh * nck + tend / ckpt_len - 1) * N * N;
#pragma unroll
                    for (int nt = 0; nt < 8; nt++)
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const int key = 16 * sw + g + (e >> 1) * 8, val = 8 * nt + 2 * tg + (e & 1);
                            p[(size_t)val * N + key] = st[nt][e];
                        }
                }
            }
            group_sync(BAR_STATE);
        }
        if (sT && !sm.abort) {
            float* p = sT + (size_t)bh * N * N;
#pragma unroll
            for (int nt = 0; nt < 8; nt++)
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int key = 16 * sw + g + (e >> 1) * 8, val = 8 * nt + 2 * tg + (e & 1);
                    p[(size_t)val * N + key] = st[nt][e];
                }
        }
    }
}

template <typename T, typename TW>
size_t smem_bytes() {
    return ((sizeof(Smem) + 127) / 128) * 128 + 2 * (size_t)Raw<T, TW>::BYTES;
}

}  // namespace ck

template <typename T, typename TW>
static int launch_fwd_chunk(const WkvFwdArgs& p, cudaStream_t st) {
    auto kern = ck::wkv7_fwd_chunk_kernel<T, TW>;
    const size_t smem = ck::smem_bytes<T, TW>();
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_cuda_error(e);
    kern<<<p.B * p.H, ck::NT, smem, st>>>((const T*)p.r, (const TW*)p.w, (const T*)p.k, (const T*)p.v,
                                          (const T*)p.a, (const T*)p.b, p.s0, (T*)p.y, p.sT, p.ckpt,
                                          p.sa, p.T, p.H, p.ckpt_len);
    return check_launch();
}

int wkv7_fwd_chunk(const WkvFwdArgs& p, cudaStream_t st) {
    RWKV_DISPATCH_DTYPE_W(p.dtype, p.w_dtype, T, TW, return launch_fwd_chunk<T, TW>(p, st));
    return RWKV_OK;
}

int read_device_error(int clear) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
    if (e != cudaSuccess) return -set_cuda_error(e);
    if (clear && v) {
        const int z = 0;
        e = cudaMemcpyToSymbol(g_device_error, &z, sizeof(int));
        if (e != cudaSuccess) return -set_cuda_error(e);
    }
    return v;
}

}  // namespace rwkv

extern "C" int rwkv_device_error(int clear) {
    const int a = rwkv::read_device_error(clear), b = rwkv::read_device_error_tc(clear),
              c = rwkv::read_device_error_bwd(clear), d = rwkv::read_device_error_moe(clear),
              e = rwkv::read_device_error_gemm(clear);
    if (a < 0) return a;
    if (b < 0) return b;
    if (c < 0) return c;
    if (d < 0) return d;
    if (e < 0) return e;
    return a | b | c | d | e;
}

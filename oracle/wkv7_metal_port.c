/*
 * CPU restatement of the reference's WKV-7 Metal kernels (test infrastructure).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load this
 * library, and only as the checker / the timed CPU baseline.  It is never the
 * product path.
 *
 * It follows rwkv_mlx/kernels/wkv7_metal.py step for step:
 *   forward  : wkv7_metal.py:28-91  (thread tid of a 64-thread threadgroup owns
 *              state row tid; snapshot every 16 steps; sa saved per step)
 *   backward : wkv7_metal.py:102-214 (reverse loop; loads the snapshot at chunk
 *              ends and otherwise reconstructs the previous state by dividing
 *              by the decay, :174-178)
 * Each Metal threadgroup becomes one (b, h) iteration of an OpenMP loop; each
 * barrier-separated phase becomes a loop over tid, so the float operations run
 * in the same order as in the kernel body.  Inputs and outputs are float32
 * (a caller with fp16 data converts before and rounds after, which is what the
 * kernel's float(x) / T(x) conversions do).
 *
 * Layouts (wkv7_metal.py:254-279): per-token tensors (B, T, H, N) row-major;
 * s = (B, H, T/16, N, N) with s[.., c, i, j] = state row i col j after step
 * 16c+15; sa = (B, T, H, N).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define WN 64
#define WCL 16

int wkv7_port_head_size(void) { return WN; }
int wkv7_port_chunk_len(void) { return WCL; }

void wkv7_port_forward(const float *r, const float *w, const float *k, const float *v,
                       const float *a, const float *b, float *y, float *s_out,
                       float *sa_out, int B, int T, int H)
{
    const int n_chunks = T / WCL;
#pragma omp parallel for schedule(static)
    for (int gid = 0; gid < B * H; gid++) {
        const int bi = gid / H, hi = gid % H;
        float state[WN][WN];
        float sh_r[WN], sh_k[WN], sh_w[WN], sh_a[WN], sh_b[WN];
        memset(state, 0, sizeof(state));
        for (int t = 0; t < T; t++) {
            const long base = (long)bi * T * H * WN + (long)t * H * WN + (long)hi * WN;
            for (int tid = 0; tid < WN; tid++) {
                sh_r[tid] = r[base + tid];
                sh_w[tid] = expf(-expf(w[base + tid]));
                sh_k[tid] = k[base + tid];
                sh_a[tid] = a[base + tid];
                sh_b[tid] = b[base + tid];
            }
            for (int tid = 0; tid < WN; tid++) {
                float *st = state[tid];
                float sa_val = 0.0f;
                for (int j = 0; j < WN; j++) sa_val += sh_a[j] * st[j];
                if (sa_out) sa_out[base + tid] = sa_val;
                const float vv = v[base + tid];
                float y_val = 0.0f;
                for (int j = 0; j < WN; j++) {
                    st[j] = st[j] * sh_w[j] + sh_k[j] * vv + sa_val * sh_b[j];
                    y_val += st[j] * sh_r[j];
                }
                y[base + tid] = y_val;
                if (s_out && (t + 1) % WCL == 0) {
                    const long cb = (((long)bi * H + hi) * n_chunks + t / WCL) * WN * WN + (long)tid * WN;
                    for (int j = 0; j < WN; j++) s_out[cb + j] = st[j];
                }
            }
        }
    }
}

void wkv7_port_backward(const float *r, const float *w, const float *k, const float *v,
                        const float *a, const float *b, const float *dy, const float *s,
                        const float *sa, float *dr, float *dw, float *dk, float *dv,
                        float *da, float *db, int B, int T, int H)
{
    const int n_chunks = T / WCL;
#pragma omp parallel for schedule(static)
    for (int gid = 0; gid < B * H; gid++) {
        const int bi = gid / H, hi = gid % H;
        /* per-thread register arrays of the kernel, indexed [tid][j] */
        static __thread float stateT[WN][WN], dstate[WN][WN], dstateT[WN][WN];
        float sh_r[WN], sh_k[WN], sh_w[WN], sh_a[WN], sh_b[WN], sh_v[WN], sh_dy[WN],
            sh_sa[WN], sh_dSb[WN];
        float wi_fac[WN], dSb_val[WN];
        memset(stateT, 0, sizeof(stateT));
        memset(dstate, 0, sizeof(dstate));
        memset(dstateT, 0, sizeof(dstateT));
        for (int t = T - 1; t >= 0; t--) {
            const long base = (long)bi * T * H * WN + (long)t * H * WN + (long)hi * WN;
            /* phase 1: stage the step's vectors (wkv7_metal.py:138-153) */
            for (int tid = 0; tid < WN; tid++) {
                wi_fac[tid] = -expf(w[base + tid]);
                sh_r[tid] = r[base + tid];
                sh_w[tid] = expf(wi_fac[tid]);
                sh_k[tid] = k[base + tid];
                sh_a[tid] = a[base + tid];
                sh_b[tid] = b[base + tid];
                sh_v[tid] = v[base + tid];
                sh_dy[tid] = dy[base + tid];
                sh_sa[tid] = sa[base + tid];
            }
            /* phase 2: per-thread gradients (wkv7_metal.py:155-200) */
            for (int tid = 0; tid < WN; tid++) {
                const float ri = sh_r[tid], wi = sh_w[tid], ki = sh_k[tid], bi_ = sh_b[tid];
                float *sT = stateT[tid], *dS = dstate[tid], *dST = dstateT[tid];
                if ((t + 1) % WCL == 0) {
                    const long cb = (((long)bi * H + hi) * n_chunks + t / WCL) * WN * WN;
                    for (int j = 0; j < WN; j++) sT[j] = s[cb + (long)j * WN + tid];
                }
                float dr_val = 0.0f;
                for (int j = 0; j < WN; j++) dr_val += sT[j] * sh_dy[j];
                dr[base + tid] = dr_val;
                const float iwi = 1.0f / wi;
                const float dyi = sh_dy[tid];
                for (int j = 0; j < WN; j++) {
                    sT[j] = (sT[j] - ki * sh_v[j] - bi_ * sh_sa[j]) * iwi;
                    dS[j] += dyi * sh_r[j];
                    dST[j] += ri * sh_dy[j];
                }
                float dw_val = 0.0f, dk_val = 0.0f, dv_val = 0.0f, db_val = 0.0f, dsb = 0.0f;
                for (int j = 0; j < WN; j++) {
                    dw_val += dST[j] * sT[j];
                    dk_val += dST[j] * sh_v[j];
                    dv_val += dS[j] * sh_k[j];
                    dsb += dS[j] * sh_b[j];
                    db_val += dST[j] * sh_sa[j];
                }
                dw[base + tid] = dw_val * wi * wi_fac[tid];
                dk[base + tid] = dk_val;
                dv[base + tid] = dv_val;
                db[base + tid] = db_val;
                dSb_val[tid] = dsb;
            }
            /* phase 3: shared dSb, da and propagation (wkv7_metal.py:197-213) */
            for (int tid = 0; tid < WN; tid++) sh_dSb[tid] = dSb_val[tid];
            for (int tid = 0; tid < WN; tid++) {
                float *sT = stateT[tid], *dS = dstate[tid], *dST = dstateT[tid];
                float da_val = 0.0f;
                for (int j = 0; j < WN; j++) da_val += sT[j] * sh_dSb[j];
                da[base + tid] = da_val;
                const float wi = sh_w[tid], ai = sh_a[tid], dsb = dSb_val[tid];
                for (int j = 0; j < WN; j++) {
                    dS[j] = dS[j] * sh_w[j] + dsb * sh_a[j];
                    dST[j] = dST[j] * wi + ai * sh_dSb[j];
                }
            }
        }
    }
}

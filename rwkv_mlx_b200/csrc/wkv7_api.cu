// C ABI entry points for WKV-7 (declared in include/rwkv_b200.h).
#include "common.cuh"
#include "wkv7.cuh"

using namespace rwkv;

namespace rwkv {
int g_wkv_impl = 0;
int g_wkv_segments = 0;  // 0: automatic segment count for the tcgen05 forward

// Segments per sequence for the tcgen05 forward: only when B*H leaves most SMs idle
// (a segment costs a transition pass, so fewer than 3 segments gains nothing), and
// with at least 8 chunks (128 steps) per segment.
static int auto_segments(int B, int T, int H) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long units = (long long)B * H;
    const int nch = (T + 15) / 16;
    if (units * 3 > sms) return 1;
    int n = (int)(sms / units);
    if (n > nch / 8) n = nch / 8;
    return n >= 3 ? n : 1;
}
static int fwd_segments(int B, int T, int H, int dtype) {
    if (!wkv7_tc_supported(dtype) || (g_wkv_impl != 0 && g_wkv_impl != 3)) return 1;
    const int nch = (T + 15) / 16;
    int n = g_wkv_segments > 0 ? g_wkv_segments : auto_segments(B, T, H);
    return n > nch ? nch : n;
}
}

static bool inputs_aligned16(const void* const* ps, int n) {
    for (int i = 0; i < n; i++)
        if (!aligned(ps[i], 16)) return false;
    return true;
}

extern "C" int rwkv_set_wkv_impl(int impl) {
    if (impl < 0 || impl > 3) return RWKV_ERR_ARG;
    g_wkv_impl = impl;
    return RWKV_OK;
}

static int check_dims(int B, int T, int H, int N, int dtype) {
    if (N != 64) return RWKV_ERR_HEAD_SIZE;
    if (B <= 0 || T <= 0 || H <= 0) return RWKV_ERR_SHAPE;
    if ((long long)B * H > 0x7fffffffLL || (long long)B * T * H * N > (1LL << 40)) return RWKV_ERR_SHAPE;
    if (dtype < RWKV_F32 || dtype > RWKV_BF16) return RWKV_ERR_DTYPE;
    return RWKV_OK;
}

static int forward_impl(const void* r, const void* w, const void* k, const void* v, const void* a,
                        const void* b, const float* s0, void* y, float* sT, float* ckpt, float* sa, int B,
                        int T, int H, int N, int dtype, int w_dtype, int ckpt_len, int nseg, void* ws,
                        size_t ws_bytes, void* stream) {
    int rc = check_dims(B, T, H, N, dtype);
    if (rc) return rc;
    if (!r || !w || !k || !v || !a || !b || !y) return RWKV_ERR_ARG;
    if (ckpt && (ckpt_len < 16 || ckpt_len % 16)) return RWKV_ERR_ARG;
    WkvFwdArgs p{r, w, k, v, a, b, s0, y, sT, ckpt, sa, B, T, H, dtype, w_dtype, ckpt ? ckpt_len : 16};
    const void* ins[6] = {r, w, k, v, a, b};
    if (g_wkv_impl == 1 || !inputs_aligned16(ins, 6)) return wkv7_fwd_seq(p, (cudaStream_t)stream);
    if (g_wkv_impl == 2) return wkv7_fwd_chunk(p, (cudaStream_t)stream);
    if (g_wkv_impl == 3 || wkv7_tc_supported(dtype)) {
        if (!wkv7_tc_supported(dtype)) return RWKV_ERR_DTYPE;
        const size_t need = wkv7_tc_ws_bytes(B, T, H, nseg);
        if (need) {
            if (!ws || ws_bytes < need) return RWKV_ERR_WORKSPACE;
            if (!aligned(ws, 16)) return RWKV_ERR_ALIGN;
        }
        return wkv7_fwd_tc(p, need ? nseg : 1, (float*)ws, (cudaStream_t)stream);
    }
    return wkv7_fwd_chunk(p, (cudaStream_t)stream);
}

extern "C" int rwkv_wkv7_forward(const void* r, const void* w, const void* k, const void* v,
                                 const void* a, const void* b, const float* s0, void* y,
                                 float* sT, float* ckpt, float* sa, int B, int T, int H, int N,
                                 int dtype, int w_dtype, int ckpt_len, void* stream) {
    return forward_impl(r, w, k, v, a, b, s0, y, sT, ckpt, sa, B, T, H, N, dtype, w_dtype, ckpt_len, 1, nullptr, 0,
                        stream);
}

extern "C" size_t rwkv_wkv7_forward_workspace_size(int B, int T, int H, int N, int dtype) {
    if (check_dims(B, T, H, N, dtype)) return 0;
    return wkv7_tc_ws_bytes(B, T, H, fwd_segments(B, T, H, dtype));
}

extern "C" int rwkv_wkv7_forward_ws(const void* r, const void* w, const void* k, const void* v,
                                    const void* a, const void* b, const float* s0, void* y,
                                    float* sT, float* ckpt, float* sa, int B, int T, int H, int N,
                                    int dtype, int w_dtype, int ckpt_len, void* workspace,
                                    size_t workspace_bytes, void* stream) {
    const int nseg = check_dims(B, T, H, N, dtype) ? 1 : fwd_segments(B, T, H, dtype);
    return forward_impl(r, w, k, v, a, b, s0, y, sT, ckpt, sa, B, T, H, N, dtype, w_dtype, ckpt_len, nseg,
                        workspace, workspace_bytes, stream);
}

extern "C" int rwkv_set_wkv_segments(int nseg) {
    if (nseg < 0) return RWKV_ERR_ARG;
    g_wkv_segments = nseg;
    return RWKV_OK;
}

extern "C" int rwkv_debug_force_wait_timeout(int on) {
    const int rc = set_force_wait_timeout_tc(on);
    return rc ? rc : set_force_wait_timeout_gemm(on);
}

extern "C" int rwkv_debug_set_device_error(int value) {
    int rc = set_device_error_tc(value);
    if (!rc) rc = set_device_error_bwd(value);
    return rc ? rc : set_device_error_gemm(value);
}

extern "C" int rwkv_wkv7_backward(const void* r, const void* w, const void* k, const void* v,
                                  const void* a, const void* b, const void* dy, const float* s0,
                                  const float* dsT, const float* ckpt, void* dr, void* dw,
                                  void* dk, void* dv, void* da, void* db, float* ds0, int B,
                                  int T, int H, int N, int dtype, int w_dtype, int ckpt_len,
                                  void* stream) {
    int rc = check_dims(B, T, H, N, dtype);
    if (rc) return rc;
    if (!r || !w || !k || !v || !a || !b || !dy || !dr || !dw || !dk || !dv || !da || !db)
        return RWKV_ERR_ARG;
    if (ckpt_len < 16 || ckpt_len % 16) return RWKV_ERR_ARG;
    if (T > ckpt_len && !ckpt) return RWKV_ERR_ARG;
    WkvBwdArgs p{r, w, k, v, a, b, dy, s0, dsT, ckpt, dr, dw, dk, dv, da, db, ds0,
                 B, T, H, dtype, w_dtype, ckpt_len};
    return wkv7_bwd_seq(p, (cudaStream_t)stream);
}

extern "C" size_t rwkv_wkv7_backward_workspace_size(int B, int T, int H, int N) {
    if (check_dims(B, T, H, N, RWKV_F32)) return 0;
    return wkv7_bwd_chunk_ws_bytes(B, T, H);
}

extern "C" int rwkv_wkv7_backward_ws(const void* r, const void* w, const void* k, const void* v,
                                     const void* a, const void* b, const void* dy, const float* s0,
                                     const float* dsT, const float* ckpt, void* dr, void* dw,
                                     void* dk, void* dv, void* da, void* db, float* ds0, int B,
                                     int T, int H, int N, int dtype, int w_dtype, int ckpt_len,
                                     void* workspace, size_t workspace_bytes, void* stream) {
    int rc = check_dims(B, T, H, N, dtype);
    if (rc) return rc;
    if (!r || !w || !k || !v || !a || !b || !dy || !dr || !dw || !dk || !dv || !da || !db)
        return RWKV_ERR_ARG;
    if (ckpt_len < 16 || ckpt_len % 16) return RWKV_ERR_ARG;
    if (T > ckpt_len && !ckpt) return RWKV_ERR_ARG;
    WkvBwdArgs p{r, w, k, v, a, b, dy, s0, dsT, ckpt, dr, dw, dk, dv, da, db, ds0,
                 B, T, H, dtype, w_dtype, ckpt_len};
    // the chunked backward needs a snapshot at every 16-step chunk boundary and reads
    // its inputs as 16-byte vectors
    const void* ins[7] = {r, w, k, v, a, b, dy};
    const bool al = inputs_aligned16(ins, 7) && aligned(ckpt, 16) && aligned(s0, 16);
    if (g_wkv_impl == 1 || ckpt_len != 16 || !al) return wkv7_bwd_seq(p, (cudaStream_t)stream);
    if (!workspace || workspace_bytes < wkv7_bwd_chunk_ws_bytes(B, T, H)) return RWKV_ERR_WORKSPACE;
    if (!aligned(workspace, 16)) return RWKV_ERR_ALIGN;
    return wkv7_bwd_chunked(p, (float*)workspace, g_wkv_segments, (cudaStream_t)stream);
}

extern "C" int rwkv_wkv7_backward_launch_count(int B, int T, int H, int N) {
    if (check_dims(B, T, H, N, RWKV_F32)) return 0;
    return wkv7_bwd_chunk_launches(B, T, H, g_wkv_segments);
}

extern "C" int rwkv_wkv7_step(float* S, const void* r, const void* w, const void* k,
                              const void* v, const void* a, const void* b, void* y, int Bs, int H,
                              int N, int dtype, int w_dtype, int w_mode, void* stream) {
    int rc = check_dims(Bs, 1, H, N, dtype);
    if (rc) return rc;
    if (!S || !r || !w || !k || !v || !a || !b || !y) return RWKV_ERR_ARG;
    if (w_mode != 0 && w_mode != 1) return RWKV_ERR_ARG;
    if (!aligned(S, 8)) return RWKV_ERR_ALIGN;
    return wkv7_step_launch(S, r, w, k, v, a, b, y, Bs, H, dtype, w_dtype, w_mode,
                            (cudaStream_t)stream);
}

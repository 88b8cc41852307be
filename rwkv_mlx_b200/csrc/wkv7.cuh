// Internal launcher interface of the WKV-7 kernels.
#pragma once
#include <cuda_runtime.h>

namespace rwkv {

struct WkvFwdArgs {
    const void *r, *w, *k, *v, *a, *b;
    const float* s0;
    void* y;
    float *sT, *ckpt, *sa;
    int B, T, H, dtype, w_dtype, ckpt_len;
};

struct WkvBwdArgs {
    const void *r, *w, *k, *v, *a, *b, *dy;
    const float *s0, *dsT, *ckpt;
    void *dr, *dw, *dk, *dv, *da, *db;
    float* ds0;
    int B, T, H, dtype, w_dtype, ckpt_len;
};

int wkv7_fwd_seq(const WkvFwdArgs& p, cudaStream_t st);
int wkv7_fwd_chunk(const WkvFwdArgs& p, cudaStream_t st);
// tcgen05 forward; nseg > 1 splits each sequence into segments run in parallel
// (transition launch + scan + forward launch), with ws of wkv7_tc_ws_bytes bytes.
int wkv7_fwd_tc(const WkvFwdArgs& p, int nseg, float* ws, cudaStream_t st);
size_t wkv7_tc_ws_bytes(int B, int T, int H, int nseg);
bool wkv7_tc_supported(int dtype);
int read_device_error_tc(int clear);
int set_force_wait_timeout_tc(int on);
int set_device_error_tc(int value);
int set_device_error_bwd(int value);
int read_device_error_bwd(int clear);
int read_device_error(int clear);
int read_device_error_moe(int clear);
// grouped tcgen05 GEMM (gemm_tc.cu): error word and test hooks
int read_device_error_gemm(int clear);
int set_force_wait_timeout_gemm(int on);
int set_device_error_gemm(int value);
extern int g_wkv_impl;  // 0 auto, 1 step-sequential, 2 chunked (mma.sync), 3 chunked (tcgen05)
int wkv7_bwd_seq(const WkvBwdArgs& p, cudaStream_t st);
size_t wkv7_bwd_chunk_ws_bytes(int B, int T, int H);
// force_nseg > 0: pass-1 segment count (tests); 0: automatic
int wkv7_bwd_chunked(const WkvBwdArgs& p, float* ws, int force_nseg, cudaStream_t st);
// kernels wkv7_bwd_chunked enqueues for these sizes on the current device
int wkv7_bwd_chunk_launches(int B, int T, int H, int force_nseg);
int wkv7_step_launch(float* S, const void* r, const void* w, const void* k, const void* v,
                     const void* a, const void* b, void* y, int Bs, int H, int dtype, int w_dtype,
                     int w_mode, cudaStream_t st);

}  // namespace rwkv

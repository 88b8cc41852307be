// Device helpers shared by the chunked WKV-7 kernels: TF32 conversion, mma.sync,
// mbarriers with bounded waits, named group barriers, cp.async, exp2, vector LDS/STS.
#pragma once
#include "common.cuh"

namespace rwkv {
namespace ck {
constexpr int N = 64, L = 16, LD4 = 68, LD8 = 72, LDM = 20;
constexpr long long WAIT_CYCLES = 4000000000LL;  // ~2 s: far above any legitimate wait

// Round to the 10-bit TF32 mantissa, ties away from zero, in two integer ops (an add
// carries into the exponent exactly as rounding up should).  Finite inputs only: the
// operands here are products of bounded activations and decay factors.
__device__ __forceinline__ uint32_t tf32(float x) {
    return (__float_as_uint(x) + 0x1000u) & 0xFFFFE000u;
}
__device__ __forceinline__ float tf32f(float x) { return __uint_as_float(tf32(x)); }
__device__ __forceinline__ uint32_t fbits(float x) { return __float_as_uint(x); }

__device__ __forceinline__ void mma8(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                     uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(unsigned long long* b, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(unsigned long long* b) {
    asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(smem_u32(b)) : "memory");
}
// Bounded wait on phase `parity`; false if it timed out or the CTA is aborting.
__device__ __forceinline__ bool mbar_wait(unsigned long long* b, uint32_t parity, volatile int* abort,
                                          int* err_word) {
    const uint32_t a = smem_u32(b);
    const long long t0 = clock64();
    while (true) {
        uint32_t ok;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
            : "=r"(ok)
            : "r"(a), "r"(parity)
            : "memory");
        if (ok) return true;
        if (*abort) return false;
        if (clock64() - t0 > WAIT_CYCLES) {
            *abort = 1;
            atomicOr(err_word, 1);
            return false;
        }
    }
}
// Bounded wait that ignores the abort flag: a CTA that is leaving waits for its own copies
// still in flight before its shared memory is released.
__device__ __forceinline__ void mbar_drain(unsigned long long* b, uint32_t parity, int* err_word) {
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
            atomicOr(err_word, 4);
            return;
        }
    }
}
// Named barrier over one warp group (128 threads) that also ORs a predicate.
__device__ __forceinline__ bool group_sync_or(int id, bool v) {
    uint32_t r;
    asm volatile(
        "{ .reg .pred p, q; setp.ne.u32 q, %1, 0; bar.red.or.pred p, %2, 128, q; selp.u32 %0, 1, 0, p; }"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void group_sync(int id) {
    asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory");
}
// Named barriers over `n` threads (a multiple of 32): wait, or wait and OR a predicate.
__device__ __forceinline__ void bar_sync_n(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ bool bar_or_n(int id, int n, bool v) {
    uint32_t r;
    asm volatile(
        "{ .reg .pred p, q; setp.ne.u32 q, %1, 0; bar.red.or.pred p, %2, %3, q; selp.u32 %0, 1, 0, p; }"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Raw input ring: per chunk, rows of r, k, v, a, b (dtype T) then w (dtype TW), each
// row padded by 16 bytes so that 16-byte reads of 8 consecutive rows hit distinct banks.
template <typename T, typename TW>
struct Raw {
    static constexpr int ROWB = N * sizeof(T), ROWBW = N * sizeof(TW);
    static constexpr int PITCH = ROWB + 16, PITCHW = ROWBW + 16;
    static constexpr int ARR = L * PITCH, ARRW = L * PITCHW;
    static constexpr int BYTES = 5 * ARR + ARRW;
    static constexpr int PPR = ROWB / 16, PPRW = ROWBW / 16;     // 16-byte pieces per row
    static constexpr int PIECES = 5 * L * PPR + L * PPRW;
    static constexpr int PER_THREAD = (PIECES + 127) / 128;
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
constexpr float LOG2E = 1.4426950408889634f;

// 8 consecutive values starting at a 16-byte aligned shared address, as floats.
template <typename T>
__device__ __forceinline__ void lds8(const unsigned char* p, float (&o)[8]) {
    if constexpr (sizeof(T) == 4) {
        const float4 x0 = *reinterpret_cast<const float4*>(p), x1 = *reinterpret_cast<const float4*>(p + 16);
        o[0] = x0.x, o[1] = x0.y, o[2] = x0.z, o[3] = x0.w, o[4] = x1.x, o[5] = x1.y, o[6] = x1.z, o[7] = x1.w;
    } else {
        const uint4 x = *reinterpret_cast<const uint4*>(p);
        const T* h = reinterpret_cast<const T*>(&x);
#pragma unroll
        for (int q = 0; q < 8; q++) o[q] = to_f32(h[q]);
    }
}
__device__ __forceinline__ void sts8(float* p, const float (&o)[8]) {
    *reinterpret_cast<float4*>(p) = make_float4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(o[4], o[5], o[6], o[7]);
}

}  // namespace ck
}  // namespace rwkv

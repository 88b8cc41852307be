// Shared helpers for the sm_100a kernels: dtype conversion, status plumbing.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "rwkv_b200.h"

namespace rwkv {

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
    return __float2bfloat16_rn(x);
}

template <typename T>
__device__ __forceinline__ float ldg_f32(const T* p) { return to_f32(__ldg(p)); }

// Record the CUDA error text for rwkv_last_error() and map to a status.
int set_cuda_error(cudaError_t e);
int check_launch();
int set_error(int code, const char* msg);  // records msg for rwkv_last_error()
void clear_error();                        // rwkv_last_error() reads "no error" again

// Internal status of the tcgen05 LoRA-MoE apply launcher: the tensor maps could not be
// built (nothing was launched), so the automatic kernel choice may fall back.
constexpr int APPLY_TC_NO_MAPS = -100;

inline bool aligned(const void* p, size_t n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }

}  // namespace rwkv

// Dispatch a templated launcher over the three dtypes.
#define RWKV_DISPATCH_DTYPE(dtype, T, ...)                 \
    switch (dtype) {                                       \
        case RWKV_F32: {                                   \
            typedef float T;                               \
            __VA_ARGS__;                                   \
            break;                                         \
        }                                                  \
        case RWKV_F16: {                                   \
            typedef __half T;                              \
            __VA_ARGS__;                                   \
            break;                                         \
        }                                                  \
        case RWKV_BF16: {                                  \
            typedef __nv_bfloat16 T;                       \
            __VA_ARGS__;                                   \
            break;                                         \
        }                                                  \
        default:                                           \
            return RWKV_ERR_DTYPE;                         \
    }

// Dispatch over (dtype, w_dtype) where w_dtype is either dtype or fp32.
#define RWKV_DISPATCH_DTYPE_W(dtype, w_dtype, T, TW, ...)          \
    RWKV_DISPATCH_DTYPE(dtype, T, {                                \
        if ((w_dtype) == (dtype)) {                                \
            typedef T TW;                                          \
            __VA_ARGS__;                                           \
        } else if ((w_dtype) == RWKV_F32) {                        \
            typedef float TW;                                      \
            __VA_ARGS__;                                           \
        } else {                                                   \
            return RWKV_ERR_DTYPE;                                 \
        }                                                          \
    })

// Chunk input staging shared by the chunked WKV-7 kernels (the tcgen05 forward and the
// backward's adjoint chain): one TMA box per input array and 16-step chunk, landed in
// shared memory with the 128-byte swizzle and read back as 8-value vectors.
//
// Box layout: 16-bit arrays as 16 rows of 64 values (row t = step, 128 bytes); fp32
// arrays as two 16-row halves of 32 values (row 16 h + t holds values 32 h .. 32 h + 31),
// because a 128-byte-swizzled box row holds at most 128 bytes.  Within a 128-byte row q,
// 16-byte piece p sits at piece p ^ (q % 8), so 16 lanes reading the same 8 values of 16
// consecutive steps hit 8 distinct bank groups (two wavefronts, the minimum for 256 B).
// The destination of every box must be 1024-byte aligned (the swizzle pattern's period);
// box_bytes() is a multiple of 1024 for every element type.
#pragma once
#include <cuda.h>

#include <type_traits>

#include "chunk_common.cuh"
#include "common.cuh"
#include "tma_common.cuh"

namespace rwkv {
namespace wst {
using ck::L;
using ck::N;

template <typename E>
constexpr int box_bytes() {
    return L * N * (int)sizeof(E);
}

__device__ __forceinline__ uint32_t swz(int q, int piece) { return (uint32_t)(q * 128 + ((piece ^ (q & 7)) << 4)); }

// values j0 .. j0 + 7 (j0 % 8 == 0) of step t of the box at `box`, as floats
template <typename E>
__device__ __forceinline__ void box8(const unsigned char* box, int t, int j0, float (&o)[8]) {
    if constexpr (sizeof(E) == 4) {
        const int q = 16 * (j0 >> 5) + t, pc = (j0 & 31) >> 2;
        const float4 x0 = *reinterpret_cast<const float4*>(box + swz(q, pc));
        const float4 x1 = *reinterpret_cast<const float4*>(box + swz(q, pc + 1));
        o[0] = x0.x, o[1] = x0.y, o[2] = x0.z, o[3] = x0.w, o[4] = x1.x, o[5] = x1.y, o[6] = x1.z, o[7] = x1.w;
    } else {
        ck::lds8<E>(box + swz(t, j0 >> 3), o);
    }
}
// value j of step t of the box at `box`
template <typename E>
__device__ __forceinline__ float box1(const unsigned char* box, int t, int j) {
    if constexpr (sizeof(E) == 4) {
        const int jj = j & 31;
        return *reinterpret_cast<const float*>(box + swz(16 * (j >> 5) + t, jj >> 2) + (jj & 3) * 4);
    } else {
        return to_f32(*reinterpret_cast<const E*>(box + swz(t, j >> 3) + (j & 7) * 2));
    }
}

// up to six input arrays' tensor maps, passed to a kernel as a __grid_constant__
struct InMaps {
    CUtensorMap m[6];
};

template <typename E>
constexpr CUtensorMapDataType map_type() {
    return sizeof(E) == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                          : (std::is_same<E, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                  : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
}

// Tensor map of one (B, T, H, 64) row-major input for the boxes above: 16-bit as
// (64, T, H, B) with a 64 x 16 box, fp32 as (32, T, 2, H, B) with a 32 x 16 x 2 box.
// Steps past T read as zero.  Returns RWKV_OK or APPLY_TC_NO_MAPS (message set).
template <typename E>
inline int make_box_map(CUtensorMap* m, const void* src, int B, int T, int H) {
    const cuuint64_t B_ = B, T_ = T, H_ = H, es = sizeof(E);
    if constexpr (sizeof(E) == 4) {
        const cuuint64_t dims[5] = {32, T_, 2, H_, B_};
        const cuuint64_t strides[4] = {H_ * N * es, 32 * es, (cuuint64_t)N * es, T_ * H_ * N * es};
        const cuuint32_t box[5] = {32, (cuuint32_t)L, 2, 1, 1};
        return tma::make_map_dt(m, map_type<E>(), src, 5, dims, strides, box, true);
    } else {
        const cuuint64_t dims[4] = {(cuuint64_t)N, T_, H_, B_};
        const cuuint64_t strides[3] = {H_ * N * es, (cuuint64_t)N * es, T_ * H_ * N * es};
        const cuuint32_t box[4] = {(cuuint32_t)N, (cuuint32_t)L, 1, 1};
        return tma::make_map_dt(m, map_type<E>(), src, 4, dims, strides, box, true);
    }
}

// Issue the box of steps tt .. tt + 15 of head hi of sequence bi; completes box_bytes<E>()
// bytes on `bar`
template <typename E>
__device__ __forceinline__ void load_box(unsigned char* dst, const CUtensorMap* m, int tt, int hi, int bi,
                                         unsigned long long* bar) {
    if constexpr (sizeof(E) == 4)
        tma::tma_load_5d(dst, m, 0, tt, 0, hi, bi, bar);
    else
        tma::tma_load_4d(dst, m, 0, tt, hi, bi, bar);
}

}  // namespace wst
}  // namespace rwkv

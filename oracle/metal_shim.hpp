// Minimal Metal-Shading-Language stand-in so that a compute-kernel BODY written
// for mx.fast.metal_kernel compiles as C++ and runs on the CPU (test
// infrastructure, never the product).
//
// One threadgroup runs at a time as real std::threads that meet at a
// std::barrier, so `threadgroup` arrays (declared static below) are shared
// between the emulated threads of the group exactly as on the GPU, and each
// threadgroup_barrier() is a real barrier.  Used by oracle/metal_cpu.py to run
// the reference's own WKV-7 kernel bodies (rwkv_mlx/kernels/wkv7_metal.py).
#pragma once
#include <barrier>
#include <cmath>
#include <cstdint>
#include <thread>
#include <vector>

typedef unsigned int uint;
typedef _Float16 half;

struct mtl_uint3 {
    uint x, y, z;
};

namespace metal {
inline float exp(float x) { return std::exp(x); }
inline float log(float x) { return std::log(x); }
inline float sqrt(float x) { return std::sqrt(x); }
inline float rsqrt(float x) { return 1.0f / std::sqrt(x); }
inline float abs(float x) { return std::fabs(x); }
inline float max(float x, float y) { return x > y ? x : y; }
inline float min(float x, float y) { return x < y ? x : y; }
}  // namespace metal

enum class mem_flags { mem_none, mem_device, mem_threadgroup };

namespace mtl_rt {
inline thread_local mtl_uint3 tpos;
inline thread_local mtl_uint3 gpos;
inline std::barrier<>* bar = nullptr;
}  // namespace mtl_rt

#define thread_position_in_threadgroup (mtl_rt::tpos)
#define threadgroup_position_in_grid (mtl_rt::gpos)
#define threadgroup static
#define device
inline void threadgroup_barrier(mem_flags) { mtl_rt::bar->arrive_and_wait(); }

// Run `body` over a Metal dispatchThreads-style launch: grid = total threads,
// tg = threads per group.  Groups run one after another.
template <class F>
inline void mtl_dispatch(uint gx, uint gy, uint gz, uint tx, uint ty, uint tz, F body) {
    const uint ngx = gx / tx, ngy = gy / ty, ngz = gz / tz;
    const uint nth = tx * ty * tz;
    for (uint gzi = 0; gzi < ngz; gzi++)
        for (uint gyi = 0; gyi < ngy; gyi++)
            for (uint gxi = 0; gxi < ngx; gxi++) {
                std::barrier<> b((std::ptrdiff_t)nth);
                mtl_rt::bar = &b;
                std::vector<std::thread> th;
                th.reserve(nth);
                for (uint tzi = 0; tzi < tz; tzi++)
                    for (uint tyi = 0; tyi < ty; tyi++)
                        for (uint txi = 0; txi < tx; txi++)
                            th.emplace_back([=]() {
                                mtl_rt::tpos = {txi, tyi, tzi};
                                mtl_rt::gpos = {gxi, gyi, gzi};
                                body();
                            });
                for (auto& t : th) t.join();
                mtl_rt::bar = nullptr;
            }
}

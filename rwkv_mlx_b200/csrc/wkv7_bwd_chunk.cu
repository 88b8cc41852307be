// WKV-7 backward, chunked (L = 16 steps per chunk), exact, in two launches.
//
// Per chunk, with X = S^T (keys x values) at the chunk start, natural-log cumulative
// decays c_t, and the decayed factors At = a e^{c_{t-1}}, Rt = r e^{c_t},
// Bh = b e^{-c_t}, Kh = k e^{-c_t}, Bb = b e^{c_L - c_t}, Kb = k e^{c_L - c_t},
// GL = e^{c_L}; Mab/Mak strictly and Mrb/Mrk inclusively lower-triangular parts of
// At Bh^T, At Kh^T, Rt Bh^T, Rt Kh^T:
//
//   U   = At X + Mab U + Mak V          (U[t] = S_{t-1} a_t, one row per step)
//   Y   = Rt X + Mrb U + Mrk V
//   X_L = GL o X + Bb^T U + Kb^T V
//
// Pass 1 (one CTA per (b, h), chunks in reverse) runs the adjoint of the state chain:
// with Inv = (I - Mab)^-1, Wu = Inv At, Wy = Rt + Mrb Wu,
//   dX_0 = GL o dX_L + Wu^T (Bb dX_L) + Wy^T dY,
// writing dX_L of every chunk to the workspace (and dX_0 of chunk 0 as ds0); two warp
// groups build Wu, Wy, Bb, dY, GL for alternating chunks while eight warps run the chain.
// Pass 2 (one CTA per (b, h, chunk), all chunks at once) forms every input gradient
// of its chunk from X (the forward's snapshot), dX_L and the inputs:
//   Lambda = Inv^T (Mrb^T dY + Bb dX_L)                 (adjoint of the solve for U)
//   dAt = Lambda X^T + dMab Bh + dMak Kh,   dMab = Lambda U^T, dMak = Lambda V^T (strict)
//   dRt = dY X^T + dMrb Bh + dMrk Kh,       dMrb = dY U^T,     dMrk = dY V^T     (incl.)
//   dBh = dMab^T At + dMrb^T Rt,  dKh = dMak^T At + dMrk^T Rt
//   dBb = U dX_L^T,  dKb = V dX_L^T,  dGL = rowsum(dX_L o X)
//   dV  = Mak^T Lambda + Mrk^T dY + Kb dX_L
// then the factor chain rule back to r, k, a, b and the reverse cumulative sum of
// the decay gradients back to w.  All products run on mma.sync: for fp32 inputs with
// operands split into high and low TF32 parts (three products, fp32-accurate), for
// 16-bit inputs as one product of TF32-rounded operands (the forward's precision;
// ~6e-4 relative error against float64 for fp16).  Chunks whose
// cumulative decay falls below e^-80 form the Mab..Mrk products and their gradients
// element-wise from exponent differences (the factored forms would overflow).
#include <algorithm>
#include <type_traits>

#include "chunk_common.cuh"
#include "common.cuh"
#include "wkv7.cuh"
#include "wkv_stage.cuh"

namespace rwkv {
namespace bwdc {
using ck::L;
using ck::N;
using ck::LD8;
using ck::mma8;
using ck::tf32;
constexpr int NT = 256;
constexpr int LDC = 68;   // row pitch (floats) of the 16x64 / 64x64 arrays
constexpr int LM = 20;    // row pitch of the 16x16 arrays
constexpr float EXT_C = -80.f;

__device__ __forceinline__ void split(float x, uint32_t& hi, uint32_t& lo) {
    hi = tf32(x);
    lo = tf32(x - __uint_as_float(hi));
}

// d (one 16x8 tile) += A(16 x K) B(K x 8); accessors take tile-local indices.  P3: split
// each operand into high and low TF32 parts (three products, fp32-accurate; used for
// fp32 inputs); otherwise one product of the TF32-rounded operands (16-bit inputs, the
// precision of the forward's TF32 products).  AX / BX: the operand's values are exactly
// representable in TF32 (16-bit inputs), so its low part is zero and the product that
// uses it is skipped.
template <bool P3, bool AX = false, bool BX = false, typename FA, typename FB>
__device__ __forceinline__ void tile_mm(float (&d)[4], const FA& A, const FB& B, int K) {
    const int lane = threadIdx.x & 31, g = lane >> 2, tg = lane & 3;
    float e[4] = {0.f, 0.f, 0.f, 0.f};   // correction terms: a separate chain from d
    float d2[4] = {0.f, 0.f, 0.f, 0.f};  // odd k-steps: a second, independent chain
    auto step = [&](int k0, float (&acc)[4]) {
        uint32_t ah[4], al[4], bh[2], bl[2];
        const float av[4] = {A(g, k0 + tg), A(g + 8, k0 + tg), A(g, k0 + tg + 4), A(g + 8, k0 + tg + 4)};
        const float bv[2] = {B(k0 + tg, g), B(k0 + tg + 4, g)};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            if (AX) ah[i] = __float_as_uint(av[i]), al[i] = 0u;
            else if (P3) split(av[i], ah[i], al[i]);
            else ah[i] = tf32(av[i]), al[i] = 0u;
        }
#pragma unroll
        for (int i = 0; i < 2; i++) {
            if (BX) bh[i] = __float_as_uint(bv[i]), bl[i] = 0u;
            else if (P3) split(bv[i], bh[i], bl[i]);
            else bh[i] = tf32(bv[i]), bl[i] = 0u;
        }
        if (P3 && !AX) mma8(e, al[0], al[1], al[2], al[3], bh[0], bh[1]);
        if (P3 && !BX) mma8(e, ah[0], ah[1], ah[2], ah[3], bl[0], bl[1]);
        mma8(acc, ah[0], ah[1], ah[2], ah[3], bh[0], bh[1]);
    };
    for (int k0 = 0; k0 < K; k0 += 16) {
        step(k0, d);
        if (k0 + 8 < K) step(k0 + 8, d2);
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        d[i] += d2[i];
        if (P3) d[i] += e[i];
    }
}
// out(m, n, v) or, when it takes a fourth argument, out(m, n, v, slot): slot 0..3 is the
// element's place in the thread's accumulator fragment (a compile-time constant at each
// call), so that results can accumulate in registers.
template <typename FO>
__device__ __forceinline__ void emit(const FO& out, int m, int n, float v, int slot) {
    if constexpr (std::is_invocable_v<FO, int, int, float, int>) out(m, n, v, slot);
    else out(m, n, v);
}
// C (M x Nn) = A (M x K) B (K x Nn) over the block's warps; out(m, n, v) once per element.
// The element -> thread mapping depends only on (M, Nn), so successive calls with the
// same shape may accumulate into the same elements without a barrier.
template <bool P3, typename FA, typename FB, typename FO>
__device__ __forceinline__ void block_mm(int M, int Nn, int K, const FA& A, const FB& B, const FO& out) {
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tg = lane & 3;
    const int ntl = Nn / 8, tiles = (M / 16) * ntl;
    for (int tile = warp; tile < tiles; tile += nw) {
        const int m0 = (tile / ntl) * 16, n0 = (tile % ntl) * 8;
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        tile_mm<P3>(d, [&](int m, int k) { return A(m0 + m, k); }, [&](int k, int n) { return B(k, n0 + n); }, K);
        emit(out, m0 + g, n0 + 2 * tg, d[0], 0);
        emit(out, m0 + g, n0 + 2 * tg + 1, d[1], 1);
        emit(out, m0 + g + 8, n0 + 2 * tg, d[2], 2);
        emit(out, m0 + g + 8, n0 + 2 * tg + 1, d[3], 3);
    }
}

// Sum of products over K segments, each with its own accessors: (A_1 B_1 + A_2 B_2 + ...)
template <bool AX_, bool BX_, typename FA, typename FB>
struct Seg {
    static constexpr bool AX = AX_, BX = BX_;
    FA A;
    FB B;
    int K;
};
template <bool AX = false, bool BX = false, typename FA, typename FB>
__device__ __forceinline__ Seg<AX, BX, FA, FB> seg(const FA& A, const FB& B, int K) {
    return Seg<AX, BX, FA, FB>{A, B, K};
}
template <bool P3, typename FO, typename... S>
__device__ __forceinline__ void block_mm_s(int M, int Nn, const FO& out, const S&... segs) {
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tg = lane & 3;
    const int ntl = Nn / 8, tiles = (M / 16) * ntl;
    for (int tile = warp; tile < tiles; tile += nw) {
        const int m0 = (tile / ntl) * 16, n0 = (tile % ntl) * 8;
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        (tile_mm<P3, S::AX, S::BX>(d, [&](int m, int k) { return segs.A(m0 + m, k); },
                               [&](int k, int n) { return segs.B(k, n0 + n); }, segs.K),
         ...);
        emit(out, m0 + g, n0 + 2 * tg, d[0], 0);
        emit(out, m0 + g, n0 + 2 * tg + 1, d[1], 1);
        emit(out, m0 + g + 8, n0 + 2 * tg, d[2], 2);
        emit(out, m0 + g + 8, n0 + 2 * tg + 1, d[3], 3);
    }
}

// nblk independent 16 x Nn products (block b: rows of A(b, m, k), B(b, k, n)), tiles
// spread over the block's warps; out(b, m, n, v) once per element.
// With `exact` set, block 1's B, block 2's A and both operands of block 3 are taken as
// exactly representable in TF32 (the layout of the stacked gradient products below).
template <bool P3, typename FA, typename FB, typename FO>
__device__ __forceinline__ void block_mm_b(int nblk, int Nn, int K, const FA& A, const FB& B, const FO& out,
                                           bool exact = false) {
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tg = lane & 3;
    const int ntl = Nn / 8, tiles = nblk * ntl;
    for (int tile = warp; tile < tiles; tile += nw) {
        const int bb = tile / ntl, n0 = (tile % ntl) * 8;
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        auto a_ = [&](int m, int k) { return A(bb, m, k); };
        auto b_ = [&](int k, int n) { return B(bb, k, n0 + n); };
        const int kind = exact ? bb : 0;
        if (kind == 1) tile_mm<P3, false, true>(d, a_, b_, K);
        else if (kind == 2) tile_mm<P3, true, false>(d, a_, b_, K);
        else if (kind == 3) tile_mm<P3, true, true>(d, a_, b_, K);
        else tile_mm<P3>(d, a_, b_, K);
        out(bb, g, n0 + 2 * tg, d[0]);
        out(bb, g, n0 + 2 * tg + 1, d[1]);
        out(bb, g + 8, n0 + 2 * tg, d[2]);
        out(bb, g + 8, n0 + 2 * tg + 1, d[3]);
    }
}

enum { IR = 0, IL, IK, IV, IA, IB, IDY, NIN };  // IL holds l = -exp(w), the natural-log decay
enum { FAT = 0, FRT, FBH, FKH, FBB, FKB, NF };

// Shared per-chunk front end: inputs -> cumulative decays -> factors -> intra-chunk
// matrices -> Inv.  `which` selects the matrices needed (bit m for Mab, Mak, Mrb, Mrk).
// The inputs other than l stay in their own type (16-bit ones are exact in fp32 and take
// half the shared memory); l = -exp(w) is fp32.
template <typename T>
struct Front {
    static constexpr int LDI = sizeof(T) == 2 ? 72 : LDC;  // conflict-free fragment reads
    T in[NIN - 1][L][LDI];
    float inl[L][LDC];
    float c[L][LDC];
    float f[NF][L][LDC];
    float GL[N];
    float M[4][L][LM];
    float Inv[L][LM];
    __device__ __forceinline__ static int slot(int arr) { return arr > IL ? arr - 1 : arr; }
    __device__ __forceinline__ float x(int arr, int t, int j) const { return to_f32(in[slot(arr)][t][j]); }
};

// One chunk's inputs: every thread issues at most one 16-byte load per array (all of
// them before any is used), then converts to fp32 into `in`.  The loads and the
// stores are split so that a caller can overlap the loads with other work.
template <typename T, typename TW>
struct ChunkLoad {
    static constexpr int VT = 16 / sizeof(T), VW = 16 / sizeof(TW);
    uint4 raw[NIN];
    __device__ __forceinline__ static int per_row(int arr) { return N / (arr == IL ? VW : VT); }
    __device__ __forceinline__ void issue(const T* r, const TW* w, const T* k, const T* v, const T* a, const T* b,
                                          const T* dy, size_t base, size_t tstride, int t0, int nt, unsigned mask) {
        const int tid = threadIdx.x;
#pragma unroll
        for (int arr = 0; arr < NIN; arr++) {
            raw[arr] = make_uint4(0, 0, 0, 0);
            const int pr = per_row(arr), row = tid / pr, col = (tid % pr) * (arr == IL ? VW : VT);
            if (!((mask >> arr) & 1) || tid >= L * pr || row >= nt) continue;
            const size_t off = base + (size_t)(t0 + row) * tstride + col;
            const void* src = arr == IR ? (const void*)(r + off) : arr == IL ? (const void*)(w + off)
                            : arr == IK ? (const void*)(k + off) : arr == IV ? (const void*)(v + off)
                            : arr == IA ? (const void*)(a + off) : arr == IB ? (const void*)(b + off)
                            : (const void*)(dy + off);
            raw[arr] = __ldg(reinterpret_cast<const uint4*>(src));
        }
    }
    __device__ __forceinline__ void store(Front<T>& fr, int nt, unsigned mask) const {
        const int tid = threadIdx.x;
#pragma unroll
        for (int arr = 0; arr < NIN; arr++) {
            const int pr = per_row(arr), row = tid / pr;
            if (!((mask >> arr) & 1) || tid >= L * pr) continue;
            if (arr == IL) {
                const TW* e = reinterpret_cast<const TW*>(&raw[arr]);
                const int col = (tid % pr) * VW;
#pragma unroll
                for (int i = 0; i < VW; i++) fr.inl[row][col + i] = row < nt ? -expf(to_f32(e[i])) : 0.f;
            } else {  // one 16-byte store (rows are 16-byte aligned: pitch LDI)
                const int col = (tid % pr) * VT;
                *reinterpret_cast<uint4*>(&fr.in[Front<T>::slot(arr)][row][col]) = raw[arr];
            }
        }
    }
};

__device__ __forceinline__ void cp16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
// 64 x 64 fp32 matrix (row-major in global memory) into smem rows of pitch LDC
__device__ __forceinline__ void cp_mat(float (*dst)[LDC], const float* src) {
    for (int e = threadIdx.x; e < N * N / 4; e += NT) cp16(&dst[e / 16][(e % 16) * 4], src + 4 * e);
}

// 4 consecutive values of a 16-bit or fp32 row in shared memory (8- / 16-byte aligned)
template <typename T>
__device__ __forceinline__ void lds4(const T* p, float (&o)[4]) {
    if constexpr (sizeof(T) == 4) {
        const float4 x = *reinterpret_cast<const float4*>(p);
        o[0] = x.x, o[1] = x.y, o[2] = x.z, o[3] = x.w;
    } else {
        const uint2 x = *reinterpret_cast<const uint2*>(p);
        const T* h = reinterpret_cast<const T*>(&x);
#pragma unroll
        for (int q = 0; q < 4; q++) o[q] = to_f32(h[q]);
    }
}
__device__ __forceinline__ void sts4(float* p, const float (&o)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(o[0], o[1], o[2], o[3]);
}
__device__ __forceinline__ float exp_(float x) { return ck::ex2(x * ck::LOG2E); }

// Cumulative decays, GL and the decayed factors: step t in lane t of a 16-lane half-warp,
// keys j0..j0+3 per thread (a shuffle scan over the steps, 16-byte row accesses).
// Returns the CTA-uniform "extreme decay" flag.
template <typename T>
__device__ int front_factors(Front<T>& fr) {
    static_assert(NT == 16 * 16, "front_factors thread layout: 16 steps x 16 groups of 4 keys");
    const int tid = threadIdx.x, lane = tid & 31, t = lane & 15, j0 = 4 * (2 * (tid >> 5) + (lane >> 4));
    float cs[4], cp[4], cl[4];
    {
        const float4 l = *reinterpret_cast<const float4*>(&fr.inl[t][j0]);
        cs[0] = l.x, cs[1] = l.y, cs[2] = l.z, cs[3] = l.w;
    }
#pragma unroll
    for (int o = 1; o < L; o <<= 1) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const float u = __shfl_up_sync(0xffffffffu, cs[q], o, 16);
            if (t >= o) cs[q] += u;
        }
    }
    int ext = 0;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const float u = __shfl_up_sync(0xffffffffu, cs[q], 1, 16);
        cp[q] = t ? u : 0.f;
        cl[q] = __shfl_sync(0xffffffffu, cs[q], L - 1, 16);
        ext |= cl[q] < EXT_C;
    }
    sts4(&fr.c[t][j0], cs);
    if (t == L - 1) {
        float gl[4];
#pragma unroll
        for (int q = 0; q < 4; q++) gl[q] = exp_(cs[q]);
        sts4(&fr.GL[j0], gl);
    }
    ext = __syncthreads_or(ext);
    float xr[4], xa[4], xb[4], xk[4], o1[4], o2[4];
    lds4<T>(&fr.in[Front<T>::slot(IR)][t][j0], xr);
    lds4<T>(&fr.in[Front<T>::slot(IA)][t][j0], xa);
    lds4<T>(&fr.in[Front<T>::slot(IB)][t][j0], xb);
    lds4<T>(&fr.in[Front<T>::slot(IK)][t][j0], xk);
#pragma unroll
    for (int q = 0; q < 4; q++) o1[q] = xa[q] * exp_(cp[q]), o2[q] = xr[q] * exp_(cs[q]);
    sts4(&fr.f[FAT][t][j0], o1);
    sts4(&fr.f[FRT][t][j0], o2);
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const float eb = exp_(cl[q] - cs[q]);
        o1[q] = xb[q] * eb, o2[q] = xk[q] * eb;
    }
    sts4(&fr.f[FBB][t][j0], o1);
    sts4(&fr.f[FKB][t][j0], o2);
    if (!ext) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const float ei = exp_(-cs[q]);
            o1[q] = xb[q] * ei, o2[q] = xk[q] * ei;
        }
        sts4(&fr.f[FBH][t][j0], o1);
        sts4(&fr.f[FKH][t][j0], o2);
    }
    __syncthreads();
    return ext;
}

// Mab, Mak (strict) and Mrb, Mrk (inclusive) for the matrices selected in `which`
template <bool P3, typename T>
__device__ void front_matrices(Front<T>& fr, int ext, unsigned which) {
    if (!ext) {
        int ms[4], nb = 0;
        for (int m = 0; m < 4; m++)
            if ((which >> m) & 1) ms[nb++] = m;
        block_mm_b<P3>(nb, L, N,
                   [&](int bb, int t, int j) { return (&fr.f[ms[bb] < 2 ? FAT : FRT][0][0])[t * LDC + j]; },
                   [&](int bb, int j, int s) { return (&fr.f[(ms[bb] & 1) ? FKH : FBH][0][0])[s * LDC + j]; },
                   [&](int bb, int t, int s, float val) {
                       const int m = ms[bb];
                       fr.M[m][t][s] = (m < 2 ? s < t : s <= t) ? val : 0.f;
                   });
    }
    for (int m = 0; m < 4; m++) {
        if (!((which >> m) & 1)) continue;
        const bool strict = m < 2;
        if (ext) {
            for (int e = threadIdx.x; e < L * L; e += NT) {
                const int t = e / L, s = e % L;
                float val = 0.f;
                if (strict ? s < t : s <= t) {
                    const int xa = m < 2 ? IA : IR, ya = (m & 1) ? IK : IB;
                    const float* cx = m < 2 ? (t ? fr.c[t - 1] : nullptr) : fr.c[t];
                    for (int j = 0; j < N; j++)
                        val = fmaf(fr.x(xa, t, j) * fr.x(ya, s, j), expf((cx ? cx[j] : 0.f) - fr.c[s][j]), val);
                }
                fr.M[m][t][s] = val;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x < L) {  // Inv = (I - Mab)^-1, one column per thread
        const int cc = threadIdx.x;
        float x[L];
#pragma unroll
        for (int t = 0; t < L; t++) x[t] = t == cc ? 1.f : 0.f;
#pragma unroll
        for (int s = 0; s < L - 1; s++) {
#pragma unroll
            for (int t = s + 1; t < L; t++) x[t] = fmaf(fr.M[0][t][s], x[s], x[t]);
        }
#pragma unroll
        for (int t = 0; t < L; t++) fr.Inv[t][cc] = x[t];
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------
// Pass 1, warp-specialized.  The chain itself needs per chunk only Wu, Wy, Bb, dY and
// GL, all functions of the inputs: two "prep" groups of 4 warps build them for
// alternating chunks into a 3-stage ring (each chunk's r, a, b, dy and w arrive as five
// TMA boxes one own chunk ahead and are read from that staging in their own type), while
// 8 "chain" warps run
// dX_0 = GL o dX_L + Wu^T (Bb dX_L) + Wy^T dY.
// Wu = (I - Mab)^-1 At comes from a forward substitution in fp32 (one key column per
// thread); the products run on mma.sync at the input type's precision (tile_mm).
namespace p1 {
constexpr int NTH = 512, NSTAGE = 3, NCW = 8;  // 8 chain warps, then two prep groups of 4 warps
enum { BAR_CHAIN = 1, BAR_PREP0 = 2 };
struct Stage {  // WU, WY are read as transposed operands: row pitch LD8 (conflict-free fragments)
    float WU[L][LD8], WY[L][LD8], BB[L][LDC], DY[L][LDC];
    float GL[N];
};
template <typename T, typename TW>
struct RawIn {  // one chunk's inputs as the TMA boxes land them (wkv_stage.cuh): r, a, b, dy, then w
    static constexpr int ARR = wst::box_bytes<T>();
    static constexpr int BYTES = 4 * ARR + wst::box_bytes<TW>();  // a multiple of 1024
};
struct Prep {
    float c[L][LDC];  // cumulative natural-log decays (read by the extreme-decay path)
    float At[L][LDC], Rt[L][LDC], Bh[L][LDC];
    float M[2][L][LM];  // Mab (strict), Mrb (inclusive)
};
struct Warps {
    int w, n;  // this warp's index within its group, warps in the group
};

// C (M x Nn) = sum over segments A_i B_i, tiles over the group's warps (see block_mm_s)
template <bool P3, typename FO, typename... S>
__device__ __forceinline__ void gmm(Warps wp, int M, int Nn, const FO& out, const S&... segs) {
    const int lane = threadIdx.x & 31, g = lane >> 2, tg = lane & 3;
    const int ntl = Nn / 8, tiles = (M / 16) * ntl;
    for (int tile = wp.w; tile < tiles; tile += wp.n) {
        const int m0 = (tile / ntl) * 16, n0 = (tile % ntl) * 8;
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        (tile_mm<P3, S::AX, S::BX>(d, [&](int m, int k) { return segs.A(m0 + m, k); },
                               [&](int k, int n) { return segs.B(k, n0 + n); }, segs.K),
         ...);
        out(m0 + g, n0 + 2 * tg, d[0]);
        out(m0 + g, n0 + 2 * tg + 1, d[1]);
        out(m0 + g + 8, n0 + 2 * tg, d[2]);
        out(m0 + g + 8, n0 + 2 * tg + 1, d[3]);
    }
}

// d[nt] (NTL adjacent 16x8 tiles) += A(16 x K) B(K x 8 NTL): each k-step's A fragment is
// loaded and rounded once for the NTL tiles, and the NTL accumulators are independent
// chains (see tile_mm for P3 / AX / BX; e holds the correction terms when P3).
template <bool P3, bool AX, bool BX, int NTL, typename FA, typename FB>
__device__ __forceinline__ void strip_mm(float (&d)[NTL][4], float (&e)[NTL][4], const FA& A, const FB& B, int K) {
    const int lane = threadIdx.x & 31, g = lane >> 2, tg = lane & 3;
    for (int k0 = 0; k0 < K; k0 += 8) {
        uint32_t ah[4], al[4];
        const float av[4] = {A(g, k0 + tg), A(g + 8, k0 + tg), A(g, k0 + tg + 4), A(g + 8, k0 + tg + 4)};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            if (AX) ah[i] = __float_as_uint(av[i]), al[i] = 0u;
            else if (P3) split(av[i], ah[i], al[i]);
            else ah[i] = tf32(av[i]), al[i] = 0u;
        }
#pragma unroll
        for (int nt = 0; nt < NTL; nt++) {
            uint32_t bh[2], bl[2];
            const float bv[2] = {B(k0 + tg, 8 * nt + g), B(k0 + tg + 4, 8 * nt + g)};
#pragma unroll
            for (int i = 0; i < 2; i++) {
                if (BX) bh[i] = __float_as_uint(bv[i]), bl[i] = 0u;
                else if (P3) split(bv[i], bh[i], bl[i]);
                else bh[i] = tf32(bv[i]), bl[i] = 0u;
            }
            if (P3 && !AX) mma8(e[nt], al[0], al[1], al[2], al[3], bh[0], bh[1]);
            if (P3 && !BX) mma8(e[nt], ah[0], ah[1], ah[2], ah[3], bl[0], bl[1]);
            mma8(d[nt], ah[0], ah[1], ah[2], ah[3], bh[0], bh[1]);
        }
    }
}
// gmm with each warp computing a strip of NTL adjacent tiles of one 16-row block
// (Nn a multiple of 8 NTL); out(m, n, v) once per element.
template <bool P3, int NTL, typename FO, typename... S>
__device__ __forceinline__ void gmm_strip(Warps wp, int M, int Nn, const FO& out, const S&... segs) {
    const int lane = threadIdx.x & 31, g = lane >> 2, tg = lane & 3;
    const int nst = Nn / (8 * NTL), strips = (M / 16) * nst;
    for (int sp = wp.w; sp < strips; sp += wp.n) {
        const int m0 = (sp / nst) * 16, n0 = (sp % nst) * 8 * NTL;
        float d[NTL][4], e[NTL][4];
#pragma unroll
        for (int nt = 0; nt < NTL; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) d[nt][i] = 0.f, e[nt][i] = 0.f;
        (strip_mm<P3, S::AX, S::BX, NTL>(d, e, [&](int m, int k) { return segs.A(m0 + m, k); },
                                         [&](int k, int n) { return segs.B(k, n0 + n); }, segs.K),
         ...);
#pragma unroll
        for (int nt = 0; nt < NTL; nt++) {
            if (P3) {
#pragma unroll
                for (int i = 0; i < 4; i++) d[nt][i] += e[nt][i];
            }
            const int n = n0 + 8 * nt + 2 * tg;
            out(m0 + g, n, d[nt][0]);
            out(m0 + g, n + 1, d[nt][1]);
            out(m0 + g + 8, n, d[nt][2]);
            out(m0 + g + 8, n + 1, d[nt][3]);
        }
    }
}

}  // namespace p1

template <typename T, typename TW, bool TR>
struct P1WSmem {
    // D and DU are read as B operands: a row pitch of 8 mod 32 floats (conflict-free
    // fragments).  The transition pass (TR) carries 128 value columns: [C | M].
    static constexpr int DC = TR ? 2 * N : N, DP = TR ? 2 * N + 8 : LD8;
    p1::Stage st[p1::NSTAGE];
    p1::Prep pg[2];
    float D[N][DP];  // dX_L [key][value]
    float DU[L][DP];
    unsigned long long full[p1::NSTAGE], empty[p1::NSTAGE];
    unsigned long long ld_full[2];  // a prep group's input boxes have landed
    int abort;
};
// dynamic shared memory of pass 1: the struct, then (1024-byte aligned) the two groups' staging
template <typename T, typename TW, bool TR>
constexpr size_t p1_smem_bytes() {
    return sizeof(P1WSmem<T, TW, TR>) + 1024 + 2 * (size_t)p1::RawIn<T, TW>::BYTES;
}

__device__ int g_device_error_bwd;

// MODE: P1_PLAIN runs chunks c_hi0 - 1 down to c_lo0 (the whole sequence, or one part of
// it: the adjoint state enters through dxl[c_hi - 1] and leaves through dxl[c_lo - 1]
// between parts).  Segmented (blockIdx.y = segment s of seg_len chunks, the top segment
// taking the remainder): P1_TRANS runs segments s >= 1 from the augmented state
// [0 | I] (64 x 128) and stores the segment's affine map D_out = M D_in + C as C into
// dxl[lo] and M into dxl[lo + 1]; P1_FINAL runs every segment from the state the scan
// left in dxl[hi - 1] (dsT for the top segment) and writes dX_L of its chunks.
enum { P1_PLAIN = 0, P1_TRANS = 1, P1_FINAL = 2 };
template <typename T, typename TW, int MODE>
__global__ void __launch_bounds__(p1::NTH, 1)
    wkv7_bwd_chain_ws_kernel(const float* __restrict__ dsT, float* __restrict__ dxl, float* __restrict__ ds0, int T_,
                             int H, int c_lo0, int c_hi0, int seg_len, const __grid_constant__ wst::InMaps maps) {
    // maps.m[0..4]: r, a, b, dy (T) and w (TW), as wst::make_box_map builds them
    using namespace p1;
    using RI = RawIn<T, TW>;
    constexpr bool TR = MODE == P1_TRANS;
    using SM = P1WSmem<T, TW, TR>;
    extern __shared__ __align__(16) unsigned char smem_p1w[];
    SM& sm = *reinterpret_cast<SM*>(smem_p1w);
    unsigned char* rawbuf = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_p1w) + sizeof(SM) + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, warp = tid >> 5, bh = blockIdx.x, bi = bh / H, hi = bh % H;
    const int nch = (T_ + L - 1) / L, nsegs = MODE == P1_PLAIN ? 1 : nch / seg_len;
    const int sg = MODE == P1_TRANS ? (int)blockIdx.y + 1 : (int)blockIdx.y;
    const int c_lo = MODE == P1_PLAIN ? c_lo0 : sg * seg_len;
    const int c_hi = MODE == P1_PLAIN ? c_hi0 : (sg == nsegs - 1 ? nch : c_lo + seg_len);
    const int cnt = c_hi - c_lo;
    constexpr bool EXI = sizeof(T) == 2;  // 16-bit dy is exact in TF32
    constexpr bool P3 = !EXI;             // three-term TF32 products for fp32 inputs

    if (tid == 0) {
        for (int i = 0; i < NSTAGE; i++) ck::mbar_init(&sm.full[i], 128), ck::mbar_init(&sm.empty[i], 32 * NCW);
        ck::mbar_init(&sm.ld_full[0], 1), ck::mbar_init(&sm.ld_full[1], 1);
        sm.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp >= NCW) {
        // ===================== prep groups =====================
        const int g_ = (warp - NCW) >> 2, pt = tid - 32 * NCW - 128 * g_, lane = pt & 31;
        const Warps wp{pt >> 5, 4};
        const int BAR = BAR_PREP0 + g_;
        Prep& pg = sm.pg[g_];
        unsigned char* raw = rawbuf + (size_t)g_ * RI::BYTES;
        // the inputs of processing index ii (chunk c_hi - 1 - ii): five TMA boxes issued by
        // lane 0 of the group's warp 3 (no share of the forward substitution); the group's
        // k-th chunk completes phase k of ld_full[g_]
        constexpr int ISSUER = 96;
        if (pt == ISSUER) {
#pragma unroll
            for (int i = 0; i < 5; i++)
                asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.m[i])) : "memory");
        }
        auto issue = [&](int ii) {
            if (pt == ISSUER) {
                tcc::proxy_fence();  // the group's generic reads of the staging precede the TMA writes
                tma::expect_tx(&sm.ld_full[g_], RI::BYTES);
                const int tt = (c_hi - 1 - ii) * L;
#pragma unroll
                for (int i = 0; i < 4; i++) wst::load_box<T>(raw + i * RI::ARR, &maps.m[i], tt, hi, bi, &sm.ld_full[g_]);
                wst::load_box<TW>(raw + 4 * RI::ARR, &maps.m[4], tt, hi, bi, &sm.ld_full[g_]);
            }
        };
        int n_issued = 0, n_used = 0;
        if (g_ < cnt) issue(g_), n_issued++;
        for (int i = g_; i < cnt; i += 2) {
            bool bad = !ck::mbar_wait(&sm.ld_full[g_], n_used & 1, &sm.abort, &g_device_error_bwd);
            if (!bad) n_used++;
            const int s = i % NSTAGE, c = c_hi - 1 - i, nt = min(L, T_ - c * L);
            Stage& stg = sm.st[s];
            if (!bad && i >= NSTAGE) bad = !ck::mbar_wait(&sm.empty[s], ((i / NSTAGE) + 1) & 1, &sm.abort, &g_device_error_bwd);
            if (ck::group_sync_or(BAR, bad)) break;
            // cumulative natural-log decays c_t = sum_{s <= t} -exp(w_s): step t in lane t of a
            // 16-lane half-warp, keys j0..j0+7 per thread, a shuffle scan over the steps
            // (rows past the sequence end are zero in the staging: their decay is 1)
            const int t = lane & 15, j0 = 8 * (2 * wp.w + (lane >> 4));
            const bool tok = t < nt;
            float wv[8], cs[8], cp[8], cl[8];
            wst::box8<TW>(raw + 4 * RI::ARR, t, j0, wv);
#pragma unroll
            for (int q = 0; q < 8; q++) cs[q] = tok ? -ck::ex2(wv[q] * ck::LOG2E) : 0.f;
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
                ext |= cl[q] < EXT_C;
            }
            ck::sts8(&pg.c[t][j0], cs);
            if (t == L - 1) {
                float gl[8];
#pragma unroll
                for (int q = 0; q < 8; q++) gl[q] = ck::ex2(cs[q] * ck::LOG2E);
                ck::sts8(&stg.GL[j0], gl);
            }
            const bool extg = ck::group_sync_or(BAR, ext);
            // decayed factors; Bb and dY go straight to the stage
            {
                float xr[8], xa[8], xb[8], xd[8], o1[8], o2[8];
                wst::box8<T>(raw + 0 * RI::ARR, t, j0, xr);
                wst::box8<T>(raw + 1 * RI::ARR, t, j0, xa);
                wst::box8<T>(raw + 2 * RI::ARR, t, j0, xb);
                wst::box8<T>(raw + 3 * RI::ARR, t, j0, xd);
#pragma unroll
                for (int q = 0; q < 8; q++)
                    o1[q] = xa[q] * ck::ex2(cp[q] * ck::LOG2E), o2[q] = xr[q] * ck::ex2(cs[q] * ck::LOG2E);
                ck::sts8(&pg.At[t][j0], o1);
                ck::sts8(&pg.Rt[t][j0], o2);
#pragma unroll
                for (int q = 0; q < 8; q++) o1[q] = xb[q] * ck::ex2((cl[q] - cs[q]) * ck::LOG2E);
                ck::sts8(&stg.BB[t][j0], o1);
                if (!extg) {
#pragma unroll
                    for (int q = 0; q < 8; q++) o2[q] = xb[q] * ck::ex2(-cs[q] * ck::LOG2E);
                    ck::sts8(&pg.Bh[t][j0], o2);
                }
                ck::sts8(&stg.DY[t][j0], xd);
            }
            ck::group_sync(BAR);
            // Mab (strict) and Mrb (inclusive): 4 tiles of 16 x 8, one per warp
            if (!extg) {
                const int which = wp.w >> 1, n0 = (wp.w & 1) * 8, g = lane >> 2, tg = lane & 3;
                float d[4] = {0.f, 0.f, 0.f, 0.f};
                const float(*X)[LDC] = which ? pg.Rt : pg.At;
                tile_mm<P3>(d, [&](int m, int k) { return X[m][k]; }, [&](int k, int n) { return pg.Bh[n0 + n][k]; }, N);
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int tt = g + (q >> 1) * 8, ss = n0 + 2 * tg + (q & 1);
                    pg.M[which][tt][ss] = (which ? ss <= tt : ss < tt) ? d[q] : 0.f;
                }
            } else {  // from exponent differences: the factored forms would overflow
                for (int e = pt; e < 2 * L * L; e += 128) {
                    const int which = e / (L * L), tt = (e / L) % L, ss = e % L;
                    float val = 0.f;
                    if (which ? ss <= tt : ss < tt) {
                        const float* cx = which ? pg.c[tt] : (tt ? pg.c[tt - 1] : nullptr);
                        for (int j = 0; j < N; j++)
                            val = fmaf(wst::box1<T>(raw + (which ? 0 : 1) * RI::ARR, tt, j) * wst::box1<T>(raw + 2 * RI::ARR, ss, j),
                                   expf((cx ? cx[j] : 0.f) - pg.c[ss][j]), val);
                    }
                    pg.M[which][tt][ss] = val;
                }
            }
            ck::group_sync(BAR);
            if (i + 2 < cnt) issue(i + 2), n_issued++;  // the raw staging is free again
            // Wu = (I - Mab)^-1 At by forward substitution, one key column per thread, in
            // blocks of 4 rows: the earlier blocks' terms of the 4 rows are 4 independent
            // chains, Mab rows are read as 16-byte vectors (same summation order per row)
            if (pt < N) {
                float x[L];
#pragma unroll
                for (int tb = 0; tb < L; tb += 4) {
                    float acc[4];
#pragma unroll
                    for (int r = 0; r < 4; r++) acc[r] = pg.At[tb + r][pt];
#pragma unroll
                    for (int q = 0; q < tb / 4; q++) {
#pragma unroll
                        for (int r = 0; r < 4; r++) {
                            const float4 m = *reinterpret_cast<const float4*>(&pg.M[0][tb + r][4 * q]);
                            acc[r] = fmaf(m.x, x[4 * q], acc[r]);
                            acc[r] = fmaf(m.y, x[4 * q + 1], acc[r]);
                            acc[r] = fmaf(m.z, x[4 * q + 2], acc[r]);
                            acc[r] = fmaf(m.w, x[4 * q + 3], acc[r]);
                        }
                    }
                    float4 md[4];
#pragma unroll
                    for (int r = 1; r < 4; r++) md[r] = *reinterpret_cast<const float4*>(&pg.M[0][tb + r][tb]);
                    x[tb] = acc[0];
                    x[tb + 1] = fmaf(md[1].x, x[tb], acc[1]);
                    x[tb + 2] = fmaf(md[2].y, x[tb + 1], fmaf(md[2].x, x[tb], acc[2]));
                    x[tb + 3] = fmaf(md[3].z, x[tb + 2], fmaf(md[3].y, x[tb + 1], fmaf(md[3].x, x[tb], acc[3])));
#pragma unroll
                    for (int r = 0; r < 4; r++) stg.WU[tb + r][pt] = x[tb + r];
                }
            }
            ck::group_sync(BAR);
            // Wy = Rt + Mrb Wu
            gmm_strip<P3, 2>(wp, L, N, [&](int t, int j, float val) { stg.WY[t][j] = pg.Rt[t][j] + val; },
                seg([&](int t, int s2) { return pg.M[1][t][s2]; }, [&](int s2, int j) { return stg.WU[s2][j]; }, L));
            ck::mbar_arrive(&sm.full[s]);
        }
        // a box issued but never waited for (the loop was left early) must land before the
        // shared memory is released
        if (pt == ISSUER && n_issued > n_used) ck::mbar_drain(&sm.ld_full[g_], (n_issued - 1) & 1, &g_device_error_bwd);
    } else {
        // ===================== chain warps =====================
        const Warps wp{warp, NCW};
        if constexpr (TR) {  // [C | M] = [0 | I]
            for (int e = tid; e < N * 2 * N; e += 32 * NCW) {
                const int j = e / (2 * N), vv = e % (2 * N);
                sm.D[j][vv] = vv == N + j ? 1.f : 0.f;
            }
        } else if (c_hi == nch) {
            for (int e = tid; e < N * N; e += 32 * NCW) {  // D = dsT^T
                const int vv = e / N, j = e % N;
                sm.D[j][vv] = dsT ? dsT[(size_t)bh * N * N + e] : 0.f;
            }
        } else {  // the adjoint state left by the part above (row-major D)
            const float* in = dxl + ((size_t)bh * nch + c_hi - 1) * N * N;
            for (int e = tid; e < N * N; e += 32 * NCW) sm.D[e / N][e % N] = in[e];
        }
        bool failed = false;
        for (int i = 0; i < cnt; i++) {
            const int c = c_hi - 1 - i, s = i % NSTAGE;
            const Stage& stg = sm.st[s];
            const bool bad = !ck::mbar_wait(&sm.full[s], (i / NSTAGE) & 1, &sm.abort, &g_device_error_bwd);
            if (ck::bar_or_n(BAR_CHAIN, 32 * NCW, bad)) {
                failed = true;
                break;
            }
#pragma unroll
            for (int hv = 0; hv < SM::DC / N; hv++) {  // DU = Bb dX_L: one 16x8 tile per warp
                // and 64 columns, its K = 64 as two independent chains
                static_assert(NCW * 8 == N, "one DU tile per chain warp");
                const int n0 = N * hv + 8 * warp, g = (tid & 31) >> 2, tg = tid & 3;
                float d0[1][4] = {}, d1[1][4] = {}, e0[1][4] = {}, e1[1][4] = {};
                strip_mm<P3, false, false, 1>(d0, e0, [&](int m, int k) { return stg.BB[m][k]; },
                                              [&](int k, int n) { return sm.D[k][n0 + n]; }, N / 2);
                strip_mm<P3, false, false, 1>(d1, e1, [&](int m, int k) { return stg.BB[m][N / 2 + k]; },
                                              [&](int k, int n) { return sm.D[N / 2 + k][n0 + n]; }, N / 2);
                float du[4];
#pragma unroll
                for (int i = 0; i < 4; i++) du[i] = (d0[0][i] + d1[0][i]) + (P3 ? e0[0][i] + e1[0][i] : 0.f);
                sm.DU[g][n0 + 2 * tg] = du[0], sm.DU[g][n0 + 2 * tg + 1] = du[1];
                sm.DU[g + 8][n0 + 2 * tg] = du[2], sm.DU[g + 8][n0 + 2 * tg + 1] = du[3];
            }
            if constexpr (!TR) {
                float* out = dxl + ((size_t)bh * nch + c) * N * N;
                for (int e = tid; e < N * N / 4; e += 32 * NCW)
                    *reinterpret_cast<float4*>(out + 4 * e) = *reinterpret_cast<const float4*>(&sm.D[e / 16][(e % 16) * 4]);
            }
            ck::bar_sync_n(BAR_CHAIN, 32 * NCW);
            gmm_strip<P3, 4>(wp, N, N, [&](int j, int vv, float val) { sm.D[j][vv] = fmaf(stg.GL[j], sm.D[j][vv], val); },
                seg([&](int j, int t) { return stg.WU[t][j]; }, [&](int t, int vv) { return sm.DU[t][vv]; }, L),
                seg<false, EXI>([&](int j, int t) { return stg.WY[t][j]; }, [&](int t, int vv) { return stg.DY[t][vv]; }, L));
            if constexpr (TR) {  // the M columns: no dY term
                gmm_strip<P3, 4>(wp, N, N, [&](int j, int vv, float val) { sm.D[j][N + vv] = fmaf(stg.GL[j], sm.D[j][N + vv], val); },
                    seg([&](int j, int t) { return stg.WU[t][j]; }, [&](int t, int vv) { return sm.DU[t][N + vv]; }, L));
            }
            ck::mbar_arrive(&sm.empty[s]);
        }
        if (failed && tid == 0) sm.abort = 1;
        ck::bar_sync_n(BAR_CHAIN, 32 * NCW);
        if constexpr (TR) {  // the segment's map: C into dxl[c_lo], M into dxl[c_lo + 1] (row-major)
            if (!failed) {
                float* oc = dxl + ((size_t)bh * nch + c_lo) * N * N;
                for (int e = tid; e < 2 * N * N / 4; e += 32 * NCW) {
                    const int half = e / (N * N / 4), q = e % (N * N / 4);
                    *reinterpret_cast<float4*>(oc + (size_t)half * N * N + 4 * q) =
                        *reinterpret_cast<const float4*>(&sm.D[q / 16][N * half + (q % 16) * 4]);
                }
            }
            return;
        }
        if (!failed && ds0 && c_lo == 0) {
            for (int e = tid; e < N * N; e += 32 * NCW) ds0[(size_t)bh * N * N + e] = sm.D[e % N][e / N];
        }
        if (!failed && c_lo > 0 && MODE == P1_PLAIN) {  // hand the adjoint state to the part below
            float* out = dxl + ((size_t)bh * nch + c_lo - 1) * N * N;
            for (int e = tid; e < N * N / 4; e += 32 * NCW)
                *reinterpret_cast<float4*>(out + 4 * e) = *reinterpret_cast<const float4*>(&sm.D[e / 16][(e % 16) * 4]);
        }
    }
}

// Segmented pass 1, between the two launches: the adjoint state entering each segment
// from above, top segment first: D_in(nsegs - 1) = dsT^T (or 0), then
// D_in(s - 1) = M_s D_in(s) + C_s with segment s's map from the transition pass, written
// to dxl[lo(s) - 1] (the top chunk slot of segment s - 1, where the final pass starts).
// The value columns are independent: eight per CTA, fp32 FMAs.
__global__ void __launch_bounds__(256)
    wkv7_bwd_seg_scan_kernel(const float* __restrict__ dsT, float* __restrict__ dxl, int nch, int seg_len) {
    __shared__ __align__(16) float Ms[2][N][LDC];  // the next segment's M lands while this one is used
    __shared__ __align__(16) float Cs[2][N][8];
    __shared__ float Din[N][8];
    const int bh = blockIdx.x, v0 = 8 * blockIdx.y, tid = threadIdx.x, k = tid >> 2, c2 = (tid & 3) * 2;
    const int nsegs = nch / seg_len;
    float* base = dxl + (size_t)bh * nch * N * N;
    auto load = [&](int sg, int buf) {  // C and M of segment sg (dxl[lo], dxl[lo + 1]), by cp.async
        const float* C = base + (size_t)(sg * seg_len) * N * N;
        const float* M = C + (size_t)N * N;
        for (int e = tid; e < N * N / 4; e += 256) cp16(&Ms[buf][e >> 4][(e & 15) * 4], M + 4 * e);
        for (int e = tid; e < N * 2; e += 256) cp16(&Cs[buf][e >> 1][4 * (e & 1)], C + (size_t)(e >> 1) * N + v0 + 4 * (e & 1));
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    for (int e = tid; e < N * 8; e += 256) {
        const int j = e >> 3, cc = e & 7;
        Din[j][cc] = dsT ? dsT[((size_t)bh * N + v0 + cc) * N + j] : 0.f;
    }
    if (nsegs >= 2) load(nsegs - 1, 0);
    for (int sg = nsegs - 1, it = 0; sg >= 1; sg--, it++) {
        const int buf = it & 1;
        if (sg >= 2) {
            load(sg - 1, buf ^ 1);  // buf ^ 1 was last read in the previous step, before its barrier
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();  // this step's M, C and the current Din visible to all
        float a0 = Cs[buf][k][c2], a1 = Cs[buf][k][c2 + 1];
#pragma unroll 8
        for (int j = 0; j < N; j++) {
            const float m = Ms[buf][k][j];
            a0 = fmaf(m, Din[j][c2], a0);
            a1 = fmaf(m, Din[j][c2 + 1], a1);
        }
        __syncthreads();  // every read of Din and of this step's buffers done
        Din[k][c2] = a0, Din[k][c2 + 1] = a1;
        float* out = base + (size_t)(sg * seg_len - 1) * N * N + (size_t)k * N + v0 + c2;
        out[0] = a0, out[1] = a1;
    }
}

int read_error_word(int clear) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_error_bwd, sizeof(int));
    if (e != cudaSuccess) return -set_cuda_error(e);
    if (clear && v) {
        const int z = 0;
        e = cudaMemcpyToSymbol(g_device_error_bwd, &z, sizeof(int));
        if (e != cudaSuccess) return -set_cuda_error(e);
    }
    return v;
}

// ---------------------------------------------------------------------------
// Pass 2: every input gradient of one chunk.  All the 16 x 64 gradient products share one
// element -> thread mapping (thread (warp w, lane g*4+tg) owns rows g, g+8 and columns
// 8w+2tg, 8w+2tg+1), so each thread accumulates its four elements of every gradient in
// registers; shared memory then fits two CTAs per SM (16-bit inputs kept 16-bit).
template <typename T>
struct P2Smem {
    Front<T> fr;
    float Sv[N][LDC];  // state at the chunk start, [value][key] (X = Sv^T); scratch at the end
    float D[N][LDC];   // dX_L, [key][value]
    float U[L][LDC], G[L][LDC];
    float Lam[L][LD8];  // read only as a B operand (row pitch LD8: conflict-free fragments)
    float dM[4][L][LM];
    float dGLp[4][N];  // partial sums of dGL over four 16-value ranges
};
struct P2Acc {  // a thread's four elements (slots) of each gradient
    float dA[4], dR[4], dB[4], dK[4], dV[4], dC[4], dCp[4], Q[4];
};

template <typename T, typename TW>
__global__ void __launch_bounds__(NT, 2)
    wkv7_bwd_chunk_kernel(const T* __restrict__ r, const TW* __restrict__ w, const T* __restrict__ k,
                          const T* __restrict__ v, const T* __restrict__ a, const T* __restrict__ b,
                          const T* __restrict__ dy, const float* __restrict__ s0, const float* __restrict__ ckpt,
                          const float* __restrict__ dxl, T* __restrict__ dr, T* __restrict__ dw, T* __restrict__ dk,
                          T* __restrict__ dv, T* __restrict__ da, T* __restrict__ db, int T_, int H, int c_off) {
    extern __shared__ __align__(16) unsigned char smem_p2[];
    P2Smem<T>& sm = *reinterpret_cast<P2Smem<T>*>(smem_p2);
    Front<T>& fr = sm.fr;
    const int tid = threadIdx.x, c = blockIdx.x + c_off, bh = blockIdx.y, bi = bh / H, hi = bh % H;
    const size_t tstride = (size_t)H * N, base = ((size_t)bi * T_ * H + hi) * N;
    const int nch = (T_ + L - 1) / L, t0 = c * L, nt = min(L, T_ - t0);
    const int lane = tid & 31, g = lane >> 2, tg = lane & 3, wrp = tid >> 5;
    auto own_t = [&](int slot) { return g + 8 * (slot >> 1); };
    auto own_j = [&](int slot) { return 8 * wrp + 2 * tg + (slot & 1); };
    P2Acc acc;
#pragma unroll
    for (int q = 0; q < 4; q++)
        acc.dA[q] = acc.dR[q] = acc.dB[q] = acc.dK[q] = acc.dV[q] = acc.dC[q] = acc.dCp[q] = acc.Q[q] = 0.f;
    // the state snapshot and dX_L by cp.async (waited for after the front below), the
    // inputs into registers; the error word is read while they are in flight
    {
        const float* S = c == 0 ? (s0 ? s0 + (size_t)bh * N * N : nullptr) : ckpt + ((size_t)bh * (T_ / L) + c - 1) * N * N;
        if (S) {
            cp_mat(sm.Sv, S);
        } else {
            for (int e = tid; e < N * LDC; e += NT) (&sm.Sv[0][0])[e] = 0.f;
        }
        cp_mat(sm.D, dxl + ((size_t)bh * nch + c) * N * N);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    ChunkLoad<T, TW> ld;
    ld.issue(r, w, k, v, a, b, dy, base, tstride, t0, nt, 0x7f);
    if (*(volatile int*)&g_device_error_bwd) {
        // pass 1 (earlier on this stream) gave up a bounded wait, so dX_L is not valid: no
        // gradient of this backward may look valid either (the word stays set until read
        // and cleared through rwkv_device_error / check_device_error)
        asm volatile("cp.async.wait_all;" ::: "memory");  // nothing may still write this CTA's shared memory
        for (int e = tid; e < nt * N; e += NT) {
            const size_t off = base + (size_t)(t0 + e / N) * tstride + (e % N);
            const T nan = from_f32<T>(__int_as_float(0x7fc00000));
            dr[off] = nan, dw[off] = nan, dk[off] = nan, dv[off] = nan, da[off] = nan, db[off] = nan;
        }
        return;
    }
    ld.store(fr, nt, 0x7f);
    __syncthreads();
    constexpr bool EXI = sizeof(T) == 2;  // 16-bit v and dy are exact in TF32
    constexpr bool P3 = !EXI;             // three-term TF32 products for fp32 inputs
    const int ext = front_factors(fr);
    front_matrices<P3>(fr, ext, 0b1111);
    const auto& F = fr.f;
    // the state snapshot and dX_L (cp.async, issued first) landed while the front ran
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();

    // U = Inv (At X + Mak V)
    block_mm_s<P3>(L, N, [&](int t, int vv, float val) { sm.G[t][vv] = val; },
               seg([&](int t, int j) { return F[FAT][t][j]; }, [&](int j, int vv) { return sm.Sv[vv][j]; }, N),
               seg<false, EXI>([&](int t, int s) { return fr.M[1][t][s]; }, [&](int s, int vv) { return fr.x(IV, s, vv); }, L));
    __syncthreads();
    block_mm<P3>(L, N, L, [&](int t, int s) { return fr.Inv[t][s]; }, [&](int s, int vv) { return sm.G[s][vv]; },
             [&](int t, int vv, float val) { sm.U[t][vv] = val; });
    // external gradient of U: Mrb^T dY + Bb dX_L
    block_mm_s<P3>(L, N, [&](int t, int vv, float val) { sm.Lam[t][vv] = val; },
               seg<false, EXI>([&](int t, int s) { return fr.M[2][s][t]; }, [&](int s, int vv) { return fr.x(IDY, s, vv); }, L),
               seg([&](int t, int j) { return F[FBB][t][j]; }, [&](int j, int vv) { return sm.D[j][vv]; }, N));
    __syncthreads();
    // Lambda = Inv^T (...)  (into G, free after U)
    block_mm<P3>(L, N, L, [&](int t, int s) { return fr.Inv[s][t]; }, [&](int s, int vv) { return sm.Lam[s][vv]; },
             [&](int t, int vv, float val) { sm.G[t][vv] = val; });
    __syncthreads();
    const auto& Lam = sm.G;
    // gradients of the intra-chunk matrices (4 stacked 16x16 products)
    block_mm_b<P3>(4, L, N,
               [&](int bb, int t, int vv) { return bb < 2 ? Lam[t][vv] : fr.x(IDY, t, vv); },
               [&](int bb, int vv, int s) { return (bb & 1) ? fr.x(IV, s, vv) : sm.U[s][vv]; },
               [&](int bb, int t, int s, float val) { sm.dM[bb][t][s] = (bb < 2 ? s < t : s <= t) ? val : 0.f; },
               EXI);
    // dV = Mak^T Lambda + Mrk^T dY + Kb dX_L
    block_mm_s<P3>(L, N, [&](int s, int vv, float val, int q) { acc.dV[q] = val; },
               seg([&](int s, int t) { return fr.M[1][t][s]; }, [&](int t, int vv) { return Lam[t][vv]; }, L),
               seg<false, EXI>([&](int s, int t) { return fr.M[3][t][s]; }, [&](int t, int vv) { return fr.x(IDY, t, vv); }, L),
               seg([&](int s, int j) { return F[FKB][s][j]; }, [&](int j, int vv) { return sm.D[j][vv]; }, N));
    {  // dGL = rowsum(dX_L o X), four threads per key (values 16 part .. 16 part + 15, rotated
       // by the key so that the reads spread over the banks); the parts are summed below
        static_assert(NT == 4 * N, "dGL thread layout");
        const int j = tid & (N - 1), part = tid >> 6;
        float sdg = 0.f;
#pragma unroll
        for (int i = 0; i < 16; i++) {
            const int vv = 16 * part + ((i + j) & 15);
            sdg = fmaf(sm.D[j][vv], sm.Sv[vv][j], sdg);
        }
        sm.dGLp[part][j] = sdg;
    }
    __syncthreads();
    // Factor gradients, accumulated in registers (same element -> thread mapping throughout).
    {
        auto outA = [&](int t, int j, float val, int q) {  // dAt: At = a e^{c_{t-1}}
            const float cp = t ? fr.c[t - 1][j] : 0.f;
            acc.dA[q] += val * exp_(cp);
            acc.dCp[q] += val * F[FAT][t][j];
        };
        auto outR = [&](int t, int j, float val, int q) {  // dRt: Rt = r e^{c_t}
            acc.dR[q] += val * exp_(fr.c[t][j]);
            acc.dC[q] += val * F[FRT][t][j];
        };
        auto sA = seg([&](int t, int vv) { return Lam[t][vv]; }, [&](int vv, int j) { return sm.Sv[vv][j]; }, N);
        auto sR = seg<EXI, false>([&](int t, int vv) { return fr.x(IDY, t, vv); }, [&](int vv, int j) { return sm.Sv[vv][j]; }, N);
        if (!ext) {
            auto bh_ = [&](int s, int j) { return F[FBH][s][j]; };
            auto kh_ = [&](int s, int j) { return F[FKH][s][j]; };
            block_mm_s<P3>(L, N, outA, sA, seg([&](int t, int s) { return sm.dM[0][t][s]; }, bh_, L),
                       seg([&](int t, int s) { return sm.dM[1][t][s]; }, kh_, L));
            block_mm_s<P3>(L, N, outR, sR, seg([&](int t, int s) { return sm.dM[2][t][s]; }, bh_, L),
                       seg([&](int t, int s) { return sm.dM[3][t][s]; }, kh_, L));
        } else {
            block_mm_s<P3>(L, N, outA, sA);
            block_mm_s<P3>(L, N, outR, sR);
        }
    }
    block_mm<P3>(L, N, N, [&](int t, int vv) { return sm.U[t][vv]; }, [&](int vv, int j) { return sm.D[j][vv]; },
             [&](int t, int j, float val, int q) {  // dBb: Bb = b e^{c_L - c_t}
                 const float qq = val * F[FBB][t][j];
                 acc.dB[q] += val * exp_(fr.c[L - 1][j] - fr.c[t][j]);
                 acc.dC[q] -= qq;
                 acc.Q[q] += qq;
             });
    block_mm_s<P3>(L, N,
               [&](int t, int j, float val, int q) {  // dKb: Kb = k e^{c_L - c_t}
                   const float qq = val * F[FKB][t][j];
                   acc.dK[q] += val * exp_(fr.c[L - 1][j] - fr.c[t][j]);
                   acc.dC[q] -= qq;
                   acc.Q[q] += qq;
               },
               seg<EXI, false>([&](int t, int vv) { return fr.x(IV, t, vv); }, [&](int vv, int j) { return sm.D[j][vv]; }, N));
    float* scr = &sm.Sv[0][0];  // Sv and D are free from here on: 2 * 64 * LDC floats of scratch
    constexpr int SA = L * LDC;  // one 16 x 64 scratch array
    if (!ext) {
        auto at = [&](int t, int j) { return F[FAT][t][j]; };
        auto rt = [&](int t, int j) { return F[FRT][t][j]; };
        block_mm_s<P3>(
            L, N,
            [&](int s, int j, float val, int q) {  // dBh = dMab^T At + dMrb^T Rt
                acc.dB[q] += val * exp_(-fr.c[s][j]);
                acc.dC[q] -= val * F[FBH][s][j];
            },
            seg([&](int s, int t) { return sm.dM[0][t][s]; }, at, L), seg([&](int s, int t) { return sm.dM[2][t][s]; }, rt, L));
        block_mm_s<P3>(
            L, N,
            [&](int s, int j, float val, int q) {  // dKh = dMak^T At + dMrk^T Rt
                acc.dK[q] += val * exp_(-fr.c[s][j]);
                acc.dC[q] -= val * F[FKH][s][j];
            },
            seg([&](int s, int t) { return sm.dM[1][t][s]; }, at, L), seg([&](int s, int t) { return sm.dM[3][t][s]; }, rt, L));
    } else {
        // element-wise: each term x_t y_s e^{c_p - c_s} (p = t-1 for Mab/Mak, t for Mrb/Mrk);
        // thread (i, j) forms the a/r terms of row i and the b/k terms of column i into
        // scratch, then every thread adds the elements it owns into its registers
        __syncthreads();
        for (int e = tid; e < L * N; e += NT) {
            const int i = e / N, j = e % N;
            const float ci = fr.c[i][j], cpi = i ? fr.c[i - 1][j] : 0.f;
            float ga = 0.f, gr = 0.f, gb = 0.f, gk = 0.f;
            for (int s = 0; s < L; s++) {
                const float cs = fr.c[s][j];
                if (s < i) ga = fmaf(sm.dM[0][i][s] * fr.x(IB, s, j) + sm.dM[1][i][s] * fr.x(IK, s, j), expf(cpi - cs), ga);
                if (s <= i) gr = fmaf(sm.dM[2][i][s] * fr.x(IB, s, j) + sm.dM[3][i][s] * fr.x(IK, s, j), expf(ci - cs), gr);
            }
            for (int t = 0; t < L; t++) {
                const float ct = fr.c[t][j], cpt = t ? fr.c[t - 1][j] : 0.f;
                if (t > i) {
                    const float e1 = expf(cpt - ci) * fr.x(IA, t, j);
                    gb = fmaf(sm.dM[0][t][i], e1, gb);
                    gk = fmaf(sm.dM[1][t][i], e1, gk);
                }
                if (t >= i) {
                    const float e2 = expf(ct - ci) * fr.x(IR, t, j);
                    gb = fmaf(sm.dM[2][t][i], e2, gb);
                    gk = fmaf(sm.dM[3][t][i], e2, gk);
                }
            }
            const int o = i * LDC + j;
            scr[0 * SA + o] = ga;
            scr[1 * SA + o] = ga * fr.x(IA, i, j);
            scr[2 * SA + o] = gr;
            scr[3 * SA + o] = gr * fr.x(IR, i, j) - gb * fr.x(IB, i, j) - gk * fr.x(IK, i, j);
            scr[4 * SA + o] = gb;
            scr[5 * SA + o] = gk;
        }
        __syncthreads();
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int o = own_t(q) * LDC + own_j(q);
            acc.dA[q] += scr[0 * SA + o];
            acc.dCp[q] += scr[1 * SA + o];
            acc.dR[q] += scr[2 * SA + o];
            acc.dC[q] += scr[3 * SA + o];
            acc.dB[q] += scr[4 * SA + o];
            acc.dK[q] += scr[5 * SA + o];
        }
    }
    __syncthreads();
    // decay: l_t = -exp(w_t); d l_tau = sum_{t >= tau} dc_t + dc_L;  dw = dl * l
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const int o = own_t(q) * LDC + own_j(q);
        scr[0 * SA + o] = acc.dC[q];
        scr[1 * SA + o] = acc.dCp[q];
        scr[2 * SA + o] = acc.Q[q];
    }
    __syncthreads();
    {  // four threads per column j, four steps each: d l_t = dc_L + suffix sum from t
        static_assert(NT == 4 * N && L == 16, "decay-gradient thread layout");
        const int j = tid & (N - 1), part = tid >> 6;
        float2* red = reinterpret_cast<float2*>(scr + 3 * SA);  // (part, column): (sum of Q, block sum)
        float suf[4], q = 0.f;
#pragma unroll
        for (int i = 3; i >= 0; i--) {
            const int t = 4 * part + i;
            q += scr[2 * SA + t * LDC + j];
            const float e = scr[0 * SA + t * LDC + j] + (t + 1 < L ? scr[1 * SA + (t + 1) * LDC + j] : 0.f);
            suf[i] = i == 3 ? e : suf[i + 1] + e;
        }
        red[part * N + j] = make_float2(q, suf[0]);
        __syncthreads();
        float dcl = ((sm.dGLp[0][j] + sm.dGLp[1][j]) + (sm.dGLp[2][j] + sm.dGLp[3][j])) * fr.GL[j], later = 0.f;
#pragma unroll
        for (int pp = 0; pp < 4; pp++) {
            const float2 r2 = red[pp * N + j];
            dcl += r2.x;
            if (pp > part) later += r2.y;
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int t = 4 * part + i;
            if (t < nt) dw[base + (size_t)(t0 + t) * tstride + j] = from_f32<T>((dcl + later + suf[i]) * fr.inl[t][j]);
        }
    }
    // the other gradients straight from registers: two adjacent columns per row
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int t = own_t(2 * h), j = own_j(2 * h);
        if (t < nt) {
            const size_t off = base + (size_t)(t0 + t) * tstride + j;
            auto st2 = [&](T* dst, float x0, float x1) {
                if constexpr (sizeof(T) == 2) {
                    T pr[2] = {from_f32<T>(x0), from_f32<T>(x1)};
                    *reinterpret_cast<uint32_t*>(dst + off) = *reinterpret_cast<const uint32_t*>(pr);
                } else {
                    *reinterpret_cast<float2*>(dst + off) = make_float2(x0, x1);
                }
            };
            st2(dr, acc.dR[2 * h], acc.dR[2 * h + 1]);
            st2(dk, acc.dK[2 * h], acc.dK[2 * h + 1]);
            st2(dv, acc.dV[2 * h], acc.dV[2 * h + 1]);
            st2(da, acc.dA[2 * h], acc.dA[2 * h + 1]);
            st2(db, acc.dB[2 * h], acc.dB[2 * h + 1]);
        }
    }
}

}  // namespace bwdc

size_t wkv7_bwd_chunk_ws_bytes(int B, int T, int H) {
    return (size_t)B * H * ((T + bwdc::L - 1) / bwdc::L) * bwdc::N * bwdc::N * sizeof(float);
}

namespace {
int sm_count() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}
// A high-priority side stream and the events that order the parts, per device and per
// calling thread (so that two host threads never interleave records of the same event).
struct PartStreams {
    static constexpr int NP = 4;
    cudaStream_t side = nullptr;
    cudaEvent_t ev[NP + 1] = {};
};
const PartStreams* part_streams() {
    thread_local PartStreams cache[16];
    thread_local bool made[16] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 16) return nullptr;
    if (!made[dev]) {
        PartStreams& c = cache[dev];
        int least = 0, greatest = 0;
        if (cudaDeviceGetStreamPriorityRange(&least, &greatest) != cudaSuccess) return nullptr;
        if (cudaStreamCreateWithPriority(&c.side, cudaStreamNonBlocking, greatest) != cudaSuccess) return nullptr;
        for (int i = 0; i <= PartStreams::NP; i++)
            if (cudaEventCreateWithFlags(&c.ev[i], cudaEventDisableTiming) != cudaSuccess) return nullptr;
        made[dev] = true;
    }
    return &cache[dev];
}
// Segmenting of pass 1 for units (b, h) chains of nch chunks: segments of seg_len chunks
// (at least 3; the top segment takes the remainder), used when nsegs >= 2.  Automatic
// when force_nseg <= 0: only when the chains leave at least three quarters of the SMs idle.
struct SegPlan {
    int seg_len, nsegs;
};
SegPlan seg_plan(int units, int nch, int force_nseg) {
    int want = force_nseg > 0 ? force_nseg : std::min(sm_count() / units, nch / 8);
    if (force_nseg <= 0 && want < 4) want = 1;
    const int seg_len = want > 1 ? std::max(3, nch / want) : nch;
    return SegPlan{seg_len, nch / seg_len};
}
bool use_parts(int units, int nch) { return sm_count() - units >= 32 && nch >= 16; }
}  // namespace

int wkv7_bwd_chunk_launches(int B, int T, int H, int force_nseg) {
    const int units = B * H, nch = (T + bwdc::L - 1) / bwdc::L;
    if (seg_plan(units, nch, force_nseg).nsegs >= 2) return 4;  // transition, scan, final, pass 2
    return use_parts(units, nch) ? 2 * PartStreams::NP : 2;
}

template <typename T, typename TW>
static int launch_bwd_chunked(const WkvBwdArgs& p, float* ws, int force_nseg, cudaStream_t st) {
    using namespace bwdc;
    auto k1 = wkv7_bwd_chain_ws_kernel<T, TW, P1_PLAIN>;
    auto k1t = wkv7_bwd_chain_ws_kernel<T, TW, P1_TRANS>;
    auto k1f = wkv7_bwd_chain_ws_kernel<T, TW, P1_FINAL>;
    auto k2 = wkv7_bwd_chunk_kernel<T, TW>;
    const int s1 = (int)p1_smem_bytes<T, TW, false>(), s1t = (int)p1_smem_bytes<T, TW, true>();
    const int s2 = (int)sizeof(P2Smem<T>);
    cudaError_t e = cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, s1);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k1t, cudaFuncAttributeMaxDynamicSharedMemorySize, s1t);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k1f, cudaFuncAttributeMaxDynamicSharedMemorySize, s1);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, s2);
    if (e != cudaSuccess) return set_cuda_error(e);
    const int nch = (p.T + L - 1) / L, units = p.B * p.H;
    alignas(64) wst::InMaps maps;  // pass 1's inputs: r, a, b, dy, w
    {
        const void* src[4] = {p.r, p.a, p.b, p.dy};
        for (int i = 0; i < 4; i++)
            if (wst::make_box_map<T>(&maps.m[i], src[i], p.B, p.T, p.H)) return RWKV_ERR_CUDA;
        if (wst::make_box_map<TW>(&maps.m[4], p.w, p.B, p.T, p.H)) return RWKV_ERR_CUDA;
    }
    auto pass1 = [&](cudaStream_t s, int lo, int hi) {
        k1<<<units, p1::NTH, s1, s>>>(p.dsT, ws, p.ds0, p.T, p.H, lo, hi, 0, maps);
        return check_launch();
    };
    auto pass2 = [&](cudaStream_t s, int lo, int hi) {
        k2<<<dim3(hi - lo, units), NT, s2, s>>>((const T*)p.r, (const TW*)p.w, (const T*)p.k, (const T*)p.v,
                                                (const T*)p.a, (const T*)p.b, (const T*)p.dy, p.s0, p.ckpt, ws,
                                                (T*)p.dr, (T*)p.dw, (T*)p.dk, (T*)p.dv, (T*)p.da, (T*)p.db, p.T,
                                                p.H, lo);
        return check_launch();
    };
    // Few (b, h) chains (at most a quarter of the SMs): pass 1 runs in segments of whole
    // chunks.  The adjoint map over a segment is affine in the state entering it from above,
    // D_out = M D_in + C (M: 64 x 64 over the keys), so a transition pass computes every
    // segment's [C | M] from [0 | I] (twice the chain's columns), a scan composes them top
    // down, and the final pass runs all segments in parallel; then pass 2 on all SMs.
    {
        const SegPlan pl = seg_plan(units, nch, force_nseg);
        const int seg_len = pl.seg_len, nsegs = pl.nsegs;
        if (nsegs >= 2) {
            k1t<<<dim3(units, nsegs - 1), p1::NTH, s1t, st>>>(p.dsT, ws, nullptr, p.T, p.H, 0, 0, seg_len, maps);
            int rc = check_launch();
            if (rc) return rc;
            wkv7_bwd_seg_scan_kernel<<<dim3(units, N / 8), 256, 0, st>>>(p.dsT, ws, nch, seg_len);
            rc = check_launch();
            if (rc) return rc;
            k1f<<<dim3(units, nsegs), p1::NTH, s1, st>>>(p.dsT, ws, p.ds0, p.T, p.H, 0, 0, seg_len, maps);
            rc = check_launch();
            return rc ? rc : pass2(st, 0, nch);
        }
    }
    // Pass 1 occupies one SM per (b, h).  When that leaves SMs idle, the chain runs in
    // parts (top chunks first) on a high-priority side stream, and pass 2 of each part
    // starts on the caller's stream as soon as its part of the chain is done, on the SMs
    // the chain leaves free.
    const PartStreams* ps = use_parts(units, nch) ? part_streams() : nullptr;
    if (!ps) {
        int rc = pass1(st, 0, nch);
        return rc ? rc : pass2(st, 0, nch);
    }
    constexpr int NP = PartStreams::NP;
    cudaError_t ce = cudaEventRecord(ps->ev[0], st);
    if (ce == cudaSuccess) ce = cudaStreamWaitEvent(ps->side, ps->ev[0], 0);
    if (ce != cudaSuccess) return set_cuda_error(ce);
    for (int q = 0; q < NP; q++) {
        const int hi = nch - (int)((long long)q * nch / NP), lo = nch - (int)((long long)(q + 1) * nch / NP);
        int rc = pass1(ps->side, lo, hi);
        if (rc) return rc;
        ce = cudaEventRecord(ps->ev[q + 1], ps->side);
        if (ce == cudaSuccess) ce = cudaStreamWaitEvent(st, ps->ev[q + 1], 0);
        if (ce != cudaSuccess) return set_cuda_error(ce);
        rc = pass2(st, lo, hi);
        if (rc) return rc;
    }
    return RWKV_OK;
}

int read_device_error_bwd(int clear) { return bwdc::read_error_word(clear); }

int set_device_error_bwd(int value) {
    return set_cuda_error(cudaMemcpyToSymbol(bwdc::g_device_error_bwd, &value, sizeof(int)));
}

int wkv7_bwd_chunked(const WkvBwdArgs& p, float* ws, int force_nseg, cudaStream_t st) {
    RWKV_DISPATCH_DTYPE_W(p.dtype, p.w_dtype, T, TW, return launch_bwd_chunked<T, TW>(p, ws, force_nseg, st));
    return RWKV_OK;
}

}  // namespace rwkv

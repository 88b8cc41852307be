// Fused LoRA-MoE adapter apply on the 5th-generation tensor cores (tcgen05) with TMA:
//
//   out = base + sum_s scores[:, s] * (x @ A[e_s]) @ B[e_s]        (rwkv_mlx/moe.py:142-147)
//
// with the E adapters concatenated: Acat = [A_0 | ... | A_{E-1}] (C x EN, EN = E * R) and
// Bcat = [B_0; ...; B_{E-1}] (EN x C).  Per tile of 128 tokens (one TMEM lane each):
//   down   D1 = X Acat            M = 128, N = EN, K = C in slices of 64 channels
//   route  H  = T(D1 * g)         g[token, e * R + r] = the token's score for expert e
//                                 (0 for experts it was not routed to), rounded to the
//                                 activation type as the reference's fp16 product is
//   up     D2 = H Bcat            M = 128, N = 64 channels per chunk, K = EN
//   out    = T(base + D2), or, when out is base, out += T(D2) by a TMA reduce-add store
//          (base is then never loaded into the SM: the add happens in L2)
//
// Data movement is all TMA, each CTA loading its own boxes: x, base and out move as
// 128-byte-swizzled 64-channel x 128-token boxes, Bcat slices as 128-byte-swizzled
// 64-channel x EN boxes (the MN-major operand layout of the up MMA), and Acat slices
// through a 4-d view of A (E, C, R) whose box lands directly in the no-swizzle MN-major
// layout of the down MMA.  The CTA is persistent over tiles and warp-specialised:
//   warp 8 lane 0   producer: one "job" (a down slice: x + Acat slices; an up chunk: Bcat +
//                   base slices) per stage of two rings, activations (NA deep: HBM) and
//                   adapter slices (NW deep: L2), armed with expect_tx;
//   warp 9 lane 0   MMA issuer: commits each job to its stages' barriers and to the up
//                   accumulator's barrier; TMEM holds two D1 accumulators (EN columns
//                   each: tiles alternate), two up accumulators of 64 columns and H
//                   (EN / 2 columns of packed 16-bit pairs, the A operand of the up MMA);
//   warps 0-7       epilogue: H per tile (TMEM -> routing scale -> TMEM), and per up chunk
//                   TMEM + base -> out in place in the activation stage (warps w and
//                   w + 4 share TMEM lanes 32 (w % 4) .. and split the columns);
//   warp 10 lane 0  store warp: TMA store (or reduce-add) of each finished out box, and
//                   release of its stage once the store has read it.
// Jobs interleave the up chunks of one tile with the down slices of the next, and a
// tile's slices start at channel block (tile mod C / 64), so that the SMs do not all
// read the same adapter slice from L2 at the same moment.
// Every wait is bounded: a wait that gives up sets the CTA's abort flag and the device
// error word, and every role leaves its loop.
#include "tma_common.cuh"

namespace rwkv {

__device__ int g_device_error_moe;  // set by a kernel that gave up a bounded wait

namespace atc {
using namespace tcc;
using namespace tma;

constexpr int TM = 128;  // tokens per tile
constexpr int KS = 64;   // channels per down slice (one 128-byte swizzle row of x)
constexpr int NC = 64;   // channels per up chunk
constexpr int NEPI = 256;       // epilogue warps 0-7: warps w and w + 4 share TMEM lanes 32 (w % 4) ..
constexpr int NTH = NEPI + 96;  // producer warp 8, MMA warp 9, store warp 10
constexpr int NA_MAX = 10, NW = 4;  // stages of the activation ring (x / base+out, <= NA_MAX) and the adapter ring
constexpr int GATE_COLS = 32;  // routed variant: the gate's two fp16 terms, 16 expert columns each
constexpr int BAR_EPI = 1;      // named barrier of the epilogue warps
constexpr int X_BYTES = TM * KS * 2;  // 128 rows x 128 bytes, swizzled
constexpr int O_BYTES = TM * NC * 2;

// RT (routed): the down product also forms the router logits, N = EN + GATE_COLS.
template <int EN, bool RT = false>
struct Geo {
    static constexpr int ENX = EN + (RT ? GATE_COLS : 0);  // N of the down product
    static constexpr int NA = RT ? 9 : 10;                  // activation stages (shared memory)
    static constexpr int A_BYTES = KS * ENX * 2;  // MN-major: K groups 128 B apart, N groups 1024 B
    static constexpr int ACAT_BYTES = KS * EN * 2;
    static constexpr int B_BYTES = EN * NC * 2;  // EN rows x 128 bytes, swizzled
    static constexpr int W_STAGE = ((A_BYTES > B_BYTES ? A_BYTES : B_BYTES) + 1023) / 1024 * 1024;
    static constexpr int A_STAGE = X_BYTES;      // = O_BYTES
    static constexpr int CTRL = 1024;
    static constexpr int SMEM = 1024 /* alignment slack */ + CTRL + NA * A_STAGE + NW * W_STAGE;
    // TMEM columns: two D1 accumulators (tiles alternate), two up accumulators, H
    static constexpr int T_D2 = 2 * ENX, T_H = 2 * ENX + 2 * NC;
    static_assert(SMEM <= 227 * 1024, "shared memory");
    static_assert(EN % 32 == 0 && T_H + EN / 2 <= 512, "TMEM columns");
    static_assert(NA <= NA_MAX, "activation ring");
};
struct Ctrl {
    unsigned long long full_a[NA_MAX], empty_a[NA_MAX];  // activation stages: landed / free
    unsigned long long full_w[NW], empty_w[NW];  // adapter stages
    unsigned long long d2_full[2], d2_empty[2];  // up-projection accumulators (double buffer)
    unsigned long long d1_full, h_full;          // down-projection done / H written
    unsigned long long out_full[2], out_empty[2];  // out box of an up chunk ready / taken by the store warp
    uint32_t tmem_base;
    int abort;
    float red_p[4][17];  // routed variant: per-warp expert probability sums (+ z), fixed order
    int red_c[4][16];    // per-warp expert counts
};
static_assert(sizeof(Ctrl) <= 1024, "control block");


// Job order of a CTA with nt tiles and n slices (= chunks) per tile: the down slices of
// tile 0, then pairs (down slice j of tile t + 1, up chunk j of tile t), then the up
// chunks of the last tile.  The up epilogues of one tile so overlap the loads and MMAs
// of the next tile's down projection (into the other D1 accumulator).
struct Job {
    bool down;
    int t, j;
};
__device__ __forceinline__ Job job_of(int g, int n, int nt) {
    if (g < n) return {true, 0, g};
    const int h = g - n, mid = (nt - 1) * 2 * n;
    if (h < mid) {
        const int pr = h >> 1;
        return (h & 1) ? Job{false, pr / n, pr % n} : Job{true, pr / n + 1, pr % n};
    }
    return {false, nt - 1, h - mid};
}
__device__ __forceinline__ int up_job_index(int t, int j, int n, int nt) {
    return t < nt - 1 ? n + t * 2 * n + 2 * j + 1 : n + (nt - 1) * 2 * n + j;
}

}  // namespace atc

// Routing outputs of the routed variant (RT): the gate operand and where the routing goes.
struct RouteArgs {
    const unsigned char* gsplit;  // gate terms, one 4 KB MN-major block per 64-channel slice
    const float* bias;            // (E,) added to the logits, or null
    int E;
    int32_t* inds;                // (ntok, topk) out
    void* scores;                 // (ntok, topk) out, activation type
    float* part_f;                // per CTA: E probability sums, then the sum of lse^2
    int32_t* part_c;              // per CTA: E counts
};

template <typename T, int EN, bool RT>
__global__ void __launch_bounds__(atc::NTH, 1)
    moe_lora_apply_tc_kernel(const __grid_constant__ CUtensorMap mx, const __grid_constant__ CUtensorMap ma,
                             const __grid_constant__ CUtensorMap mb, const __grid_constant__ CUtensorMap mbase,
                             const __grid_constant__ CUtensorMap mout, int has_base, int accum,
                             const int32_t* __restrict__ inds, const T* __restrict__ scores, int ntok, int C,
                             int R, int topk, const RouteArgs ra) {
    using namespace atc;
    using G = Geo<EN, RT>;
    constexpr int NA = G::NA;
    constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
    constexpr uint32_t IDESC_DOWN = idesc_16(TM, G::ENX, BF, false, true);
    constexpr uint32_t IDESC_UP = idesc_16(TM, NC, BF, false, true);

    extern __shared__ __align__(1024) unsigned char smem_atc_raw[];
    // the swizzled tiles need 1024-byte alignment of the shared-memory address
    const uint32_t raw_addr = ck::smem_u32(smem_atc_raw);
    unsigned char* smem = smem_atc_raw + (((raw_addr + 1023) & ~1023u) - raw_addr);
    Ctrl& cs = *reinterpret_cast<Ctrl*>(smem);
    unsigned char* ring_a = smem + G::CTRL;
    unsigned char* ring_w = ring_a + NA * G::A_STAGE;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nsl = C / KS, nch = C / NC;  // equal: KS == NC
    const int ntiles = (ntok + TM - 1) / TM;
    const int my_tiles = (int)blockIdx.x < ntiles ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int njobs = my_tiles * (nsl + nch);

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                         ck::smem_u32(&cs.tmem_base))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == NEPI) {
        for (int i = 0; i < NA; i++) ck::mbar_init(&cs.full_a[i], 1), ck::mbar_init(&cs.empty_a[i], 1);
        for (int i = 0; i < NW; i++) ck::mbar_init(&cs.full_w[i], 1), ck::mbar_init(&cs.empty_w[i], 1);
        for (int i = 0; i < 2; i++) ck::mbar_init(&cs.d2_full[i], 1), ck::mbar_init(&cs.d2_empty[i], NEPI);
        ck::mbar_init(&cs.d1_full, 1);
        ck::mbar_init(&cs.h_full, NEPI);
        for (int i = 0; i < 2; i++) ck::mbar_init(&cs.out_full[i], 1), ck::mbar_init(&cs.out_empty[i], 1);
        cs.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = cs.tmem_base;
    auto tile0 = [&](int lt) { return ((int)blockIdx.x + lt * (int)gridDim.x) * TM; };
    // Slice / chunk j of a tile's sequence is channel block (j + tile) % nsl: CTAs working
    // on neighbouring tiles at the same time then read different adapter slices, instead
    // of all SMs requesting the same few L2 lines at once.
    auto blk = [&](int lt, int j) {
        const int r = j + ((int)blockIdx.x + lt * (int)gridDim.x) % nsl;
        return r >= nsl ? r - nsl : r;
    };
    int* err = &g_device_error_moe;

    if (warp == NEPI / 32) {
        // ============ producer: TMA of job g into activation stage g % NA, adapter stage g % NW ============
        if (lane == 0) {
            for (int g = 0; g < njobs; g++) {
                const int sa = g % NA, sw = g % NW;
                if (g >= NA && !ck::mbar_wait(&cs.empty_a[sa], ((g / NA) + 1) & 1, &cs.abort, err)) break;
                if (g >= NW && !ck::mbar_wait(&cs.empty_w[sw], ((g / NW) + 1) & 1, &cs.abort, err)) break;
                const Job jb = job_of(g, nsl, my_tiles);
                const int t0 = tile0(jb.t);
                unsigned char* sta = ring_a + sa * G::A_STAGE;
                unsigned char* stw = ring_w + sw * G::W_STAGE;
                if (jb.down) {
                    expect_tx(&cs.full_w[sw], G::A_BYTES);
                    tma_load_4d(stw, &ma, 0, blk(jb.t, jb.j) * KS, 0, 0, &cs.full_w[sw]);
                    if constexpr (RT)  // the gate slice continues the N groups of the Acat slice
                        bulk_load(stw + G::ACAT_BYTES, ra.gsplit + (size_t)blk(jb.t, jb.j) * (KS * GATE_COLS * 2),
                                  KS * GATE_COLS * 2, &cs.full_w[sw]);
                    expect_tx(&cs.full_a[sa], X_BYTES);
                    tma_load_2d(sta, &mx, blk(jb.t, jb.j) * KS, t0, &cs.full_a[sa]);
                } else {
                    const int cj = blk(jb.t, jb.j) * NC;
                    expect_tx(&cs.full_w[sw], G::B_BYTES);
                    tma_load_2d(stw, &mb, cj, 0, &cs.full_w[sw]);
                    const bool ld = has_base && !accum;  // accumulating into out = base: nothing to load
                    expect_tx(&cs.full_a[sa], ld ? O_BYTES : 0);
                    if (ld) tma_load_2d(sta, &mbase, cj, t0, &cs.full_a[sa]);
                }
            }
        }
        __syncwarp();
    } else if (warp == NEPI / 32 + 1) {
        // ============ MMA issuer ============
        if (lane == 0) {
            int q = 0;  // up chunks issued so far (TMEM buffer q & 1, use q >> 1)
            for (int g = 0; g < njobs; g++) {
                const int sa = g % NA, sw = g % NW;
                const Job jb = job_of(g, nsl, my_tiles);
                if (!ck::mbar_wait(&cs.full_w[sw], (g / NW) & 1, &cs.abort, err)) break;
                if (jb.down && !ck::mbar_wait(&cs.full_a[sa], (g / NA) & 1, &cs.abort, err)) break;
                if (!jb.down && jb.j == 0 && !ck::mbar_wait(&cs.h_full, jb.t & 1, &cs.abort, err)) break;
                if (!jb.down && q >= 2 && !ck::mbar_wait(&cs.d2_empty[q & 1], ((q >> 1) + 1) & 1, &cs.abort, err))
                    break;
                tc_fence_after();
                const uint32_t stw = ck::smem_u32(ring_w + sw * G::W_STAGE);
                if (jb.down) {
                    // A = x slice (K-major, 128-byte swizzle: K step = 32 bytes within the row),
                    // B = Acat slice (MN-major, no swizzle: K groups 128 B, N groups 1024 B)
                    const uint32_t sta = ck::smem_u32(ring_a + sa * G::A_STAGE);
#pragma unroll
                    for (int kk = 0; kk < KS / 16; kk++)
                        umma16(tmem + (jb.t & 1) * G::ENX, desc_sw128(sta + kk * 32, 16, 1024),
                               umma_desc_ls(stw + kk * 256, 128, 1024), IDESC_DOWN, (jb.j > 0 || kk > 0) ? 1u : 0u);
                    umma_commit(&cs.empty_a[sa]);
                    umma_commit(&cs.empty_w[sw]);
                    if (jb.j == nsl - 1) umma_commit(&cs.d1_full);
                } else {
                    // A = H in TMEM (8 columns per K step of 16), B = Bcat slice (MN-major,
                    // 128-byte swizzle: 8 K rows of 128 bytes per 1024-byte group)
                    const uint32_t d2 = tmem + G::T_D2 + (q & 1) * NC;
#pragma unroll
                    for (int kk = 0; kk < EN / 16; kk++)
                        umma16_ts(d2, tmem + G::T_H + kk * 8, desc_sw128(stw + kk * 2048, 8192, 1024), IDESC_UP,
                                  kk > 0 ? 1u : 0u);
                    umma_commit(&cs.empty_w[sw]);
                    umma_commit(&cs.d2_full[q & 1]);
                    q++;
                }
            }
        }
        __syncwarp();
    } else if (warp == NEPI / 32 + 2) {
        // ============ store warp: out boxes -> global (TMA store, or reduce-add into out = base) ============
        if (lane == 0) {
            int q = 0, p1 = 0, p2 = 0;  // act stages of the stores of chunks q - 1, q - 2 (released once read)
            for (int lt = 0; lt < my_tiles; lt++) {
                const int t0 = tile0(lt);
                bool bad = false;
                for (int j = 0; j < nch; j++, q++) {
                    const int sa = up_job_index(lt, j, nsl, my_tiles) % NA;
                    if (!ck::mbar_wait(&cs.out_full[q & 1], (q >> 1) & 1, &cs.abort, err)) {
                        bad = true;
                        break;
                    }
                    ck::mbar_arrive(&cs.out_empty[q & 1]);
                    const unsigned char* os = ring_a + sa * G::A_STAGE;
                    if (accum)
                        tma_add_2d(&mout, blk(lt, j) * NC, t0, os);  // out (= base) += T(D2)
                    else
                        tma_store_2d(&mout, blk(lt, j) * NC, t0, os);  // rows past ntok are not written
                    bulk_wait_read<2>();  // the store of chunk q - 2 has read its box
                    if (q >= 2) ck::mbar_arrive(&cs.empty_a[p2]);
                    p2 = p1;
                    p1 = sa;
                }
                if (bad) break;
            }
            bulk_wait_all();
        }
        __syncwarp();
    } else {
        // ============ epilogue warps 0-7: H per tile, out per up chunk ============
        const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
        const int row = 32 * (warp & 3) + lane;  // token row of the tile = TMEM lane
        const int hf = warp >> 2;                // which half of the columns this thread handles
        int q = 0;                               // up chunks done (TMEM buffer q & 1)
        bool bad = false;
        float acc_p[16], acc_z = 0.f;  // routed variant: this thread's routing statistics
        int acc_c[16];
        float lbias[16];                // routed variant: the logit bias (0 past E)
#pragma unroll
        for (int e = 0; e < 16; e++) {
            acc_p[e] = 0.f, acc_c[e] = 0;
            lbias[e] = (RT && ra.bias && e < ra.E) ? ra.bias[e] : 0.f;
        }
        for (int lt = 0; lt < my_tiles && !bad; lt++) {
            const int t0 = tile0(lt), tok = t0 + row;
            {
                const int kq = tok < ntok ? topk : 0;
                int es[8];
                float ss[8];
                if constexpr (!RT) {
#pragma unroll
                    for (int s = 0; s < 8; s++) {
                        es[s] = s < kq ? inds[(size_t)tok * topk + s] : -1;
                        ss[s] = s < kq ? (scores ? to_f32(scores[(size_t)tok * topk + s]) : 1.f) : 0.f;
                    }
                }
                bad = ck::bar_or_n(BAR_EPI, NEPI, !ck::mbar_wait(&cs.d1_full, lt & 1, &cs.abort, err));
                if (bad) break;  // the vote keeps the threads together for the named barriers
                tc_fence_after();
                if constexpr (RT) {
                    // router (moe.py:56-86): logits = x W^T from the two gate terms
                    // (W = W0 + W1 / 2048, each product exact in fp32), + bias; full-softmax
                    // statistics, top-k by repeated argmax with ties to the lower expert id,
                    // softmax over the selected logits rounded to the activation type
                    float hi[16], lo[16], lg[16];
                    tmem_ld16(tmem + lane_base + (lt & 1) * G::ENX + EN, hi);
                    tmem_ld16(tmem + lane_base + (lt & 1) * G::ENX + EN + 16, lo);
                    tmem_wait_ld();
                    const int E = ra.E;
                    float m = -INFINITY;
#pragma unroll
                    for (int e = 0; e < 16; e++) {
                        lg[e] = e < E ? hi[e] + lo[e] * (1.f / 2048.f) + lbias[e] : -INFINITY;
                        m = fmaxf(m, lg[e]);
                    }
                    float ex[16], se = 0.f;
#pragma unroll
                    for (int e = 0; e < 16; e++) ex[e] = e < E ? expf(lg[e] - m) : 0.f, se += ex[e];
                    const bool tv = tok < ntok;
                    if (tv && hf == 0) {
#pragma unroll
                        for (int e = 0; e < 16; e++) acc_p[e] += ex[e] / se;
                        const float lse = m + logf(se);
                        acc_z = fmaf(lse, lse, acc_z);
                    }
                    unsigned taken = 0;
                    float sel0 = 0.f, denom = 0.f;
#pragma unroll
                    for (int s = 0; s < 8; s++) {
                        es[s] = -1;
                        if (s < kq) {
                            float bv = -INFINITY;
                            int bi = -1;
#pragma unroll
                            for (int e = 0; e < 16; e++)  // ascending ids, strictly greater: ties to the lower id
                                if (e < E && !((taken >> e) & 1u) && (bi < 0 || lg[e] > bv)) bv = lg[e], bi = e;
                            if (bi < 0) bi = 0;  // topk <= E is checked on the host
                            taken |= 1u << bi;
                            es[s] = bi;
                            ss[s] = bv;  // the logit for now
                            if (s == 0) sel0 = bv;
                            denom += expf(bv - sel0);
                        }
                    }
#pragma unroll
                    for (int s = 0; s < 8; s++) {
                        if (s < kq) {
                            const T sc = from_f32<T>(expf(ss[s] - sel0) / denom);
                            ss[s] = to_f32(sc);  // H uses the score in the activation type
                            if (hf == 0) {
                                ra.inds[(size_t)tok * topk + s] = es[s];
                                reinterpret_cast<T*>(ra.scores)[(size_t)tok * topk + s] = sc;
#pragma unroll
                                for (int e = 0; e < 16; e++) acc_c[e] += es[s] == e ? 1 : 0;
                            }
                        } else {
                            ss[s] = 0.f;
                        }
                    }
                }
#pragma unroll
                for (int h0 = hf * (EN / 2); h0 < (hf + 1) * (EN / 2); h0 += 16) {
                    float v[16];
                    uint32_t hp[8];
                    tmem_ld16(tmem + lane_base + (lt & 1) * G::ENX + h0, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 16; c += 8) {
                        const int e = (h0 + c) / R;
                        float gs = 0.f;
#pragma unroll
                        for (int s = 0; s < 8; s++) gs += es[s] == e ? ss[s] : 0.f;
#pragma unroll
                        for (int u = 0; u < 8; u += 2) {
                            T pr[2] = {from_f32<T>(v[c + u] * gs), from_f32<T>(v[c + u + 1] * gs)};
                            hp[(c + u) / 2] = *reinterpret_cast<const uint32_t*>(pr);
                        }
                    }
                    tmem_st8(tmem + lane_base + G::T_H + h0 / 2, hp);
                }
                tmem_wait_st();
                tc_fence_before();
                ck::mbar_arrive(&cs.h_full);
            }
            for (int j = 0; j < nch; j++, q++) {
                const int g = up_job_index(lt, j, nsl, my_tiles), sa = g % NA;
                unsigned char* os = ring_a + sa * G::A_STAGE;  // base slice, then out in place
                bad = !ck::mbar_wait(&cs.d2_full[q & 1], (q >> 1) & 1, &cs.abort, err) ||
                      !ck::mbar_wait(&cs.full_a[sa], (g / NA) & 1, &cs.abort, err);
                bad = ck::bar_or_n(BAR_EPI, NEPI, bad);
                if (bad) break;
                tc_fence_after();
                float v[32];
                const uint32_t ta = tmem + lane_base + G::T_D2 + (q & 1) * NC + hf * 32;
                tmem_ld16(ta, v);
                tmem_ld16(ta + 16, v + 16);
                tmem_wait_ld();
                tc_fence_before();
                ck::mbar_arrive(&cs.d2_empty[q & 1]);
                // this row of the 128-byte-swizzled base / out box: 16-byte piece c sits at c ^ (row % 8)
                unsigned char* orow = os + row * 128;
#pragma unroll
                for (int c4 = 0; c4 < 4; c4++) {
                    const int c = hf * 4 + c4;
                    unsigned char* pp = orow + ((c ^ (row & 7)) << 4);
                    uint4 raw = (has_base && !accum) ? *reinterpret_cast<const uint4*>(pp) : make_uint4(0u, 0u, 0u, 0u);
                    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
                    for (int u = 0; u < 8; u++) e[u] = from_f32<T>(v[8 * c4 + u] + to_f32(e[u]));
                    *reinterpret_cast<uint4*>(pp) = raw;
                }
                proxy_fence();  // the TMA store reads these bytes through the async proxy
                ck::bar_sync_n(BAR_EPI, NEPI);
                if (tid == 0) {  // hand the box to the store warp
                    // a wait that gives up sets the abort flag: the next wait of every epilogue
                    // thread then fails too and their vote ends the loops together
                    if (q >= 2) ck::mbar_wait(&cs.out_empty[q & 1], ((q >> 1) + 1) & 1, &cs.abort, err);
                    ck::mbar_arrive(&cs.out_full[q & 1]);
                }
            }
        }
        if constexpr (RT) {
            // this CTA's routing partials, in a fixed order: lanes, then warps 0-3
            const int E = ra.E;
            if (hf == 0) {
#pragma unroll
                for (int e = 0; e < 16; e++) {
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        acc_p[e] += __shfl_xor_sync(0xffffffffu, acc_p[e], o);
                        acc_c[e] += __shfl_xor_sync(0xffffffffu, acc_c[e], o);
                    }
                }
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) acc_z += __shfl_xor_sync(0xffffffffu, acc_z, o);
                if (lane == 0) {
#pragma unroll
                    for (int e = 0; e < 16; e++) cs.red_p[warp][e] = acc_p[e], cs.red_c[warp][e] = acc_c[e];
                    cs.red_p[warp][16] = acc_z;
                }
            }
            ck::bar_sync_n(BAR_EPI, NEPI);
            if (tid <= E) {
                const bool ab = cs.abort != 0;
                float sp = 0.f;
                int sc = 0;
                for (int w = 0; w < 4; w++) sp += cs.red_p[w][tid < E ? tid : 16], sc += tid < E ? cs.red_c[w][tid] : 0;
                ra.part_f[(size_t)blockIdx.x * (E + 1) + tid] = ab ? __int_as_float(0x7fc00000) : sp;
                if (tid < E) ra.part_c[(size_t)blockIdx.x * E + tid] = sc;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
}

// Gate operand of the routed variant: W (E, C) fp32 split into W0 = fp16(W) and
// W1 = fp16((W - W0) * 2048) (every fp16 x fp16 product is exact in fp32, so the logits
// keep fp32-level rounding), laid out per 64-channel slice as the MN-major no-swizzle
// core matrices of the down product's B operand: column n < 16 is expert n's W0,
// 16 <= n < 32 expert (n - 16)'s W1 (zero past E); N group n / 8 at 1024 bytes, K group
// (channel / 8) at 128 bytes, 16 bytes per channel.
__global__ void moe_gate_split_kernel(const float* __restrict__ W, __half* __restrict__ out, int E, int C) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;  // one (channel, column) pair
    if (i >= C * atc::GATE_COLS) return;
    const int c = i / atc::GATE_COLS, n = i % atc::GATE_COLS, e = n & 15;
    const float w = e < E ? W[(size_t)e * C + c] : 0.f;
    const __half w0 = __float2half_rn(w);
    const __half v = n < 16 ? w0 : __float2half_rn((w - __half2float(w0)) * 2048.f);
    const int s = c / atc::KS, k = c % atc::KS;
    const size_t byte = (size_t)s * atc::KS * atc::GATE_COLS * 2 + (n / 8) * 1024 + (k / 8) * 128 + (k % 8) * 16 + (n % 8) * 2;
    out[byte / 2] = v;
}

int moe_apply_tc_grid(int ntok) {
    int dev = 0, nsm = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    const int ntiles = (ntok + atc::TM - 1) / atc::TM;
    return ntiles < nsm ? ntiles : nsm;  // persistent: one CTA per SM
}

template <typename T, int EN, bool RT>
static int launch_apply_tc(const void* x, const void* base, const void* A, const void* B, const int32_t* inds,
                           const void* scores, void* out, int ntok, int C, int R, int topk, const RouteArgs& ra,
                           cudaStream_t st) {
    using namespace atc;
    constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
    const int E = EN / R, rp = R / 8;
    alignas(64) CUtensorMap mx, ma, mb, mbase, mout;
    const cuuint64_t row_stride[1] = {(cuuint64_t)C * 2};
    {  // x, base, out: (ntok, C) row-major; box 64 channels x 128 tokens, 128-byte swizzle
        const cuuint64_t dims[2] = {(cuuint64_t)C, (cuuint64_t)ntok};
        const cuuint32_t box[2] = {(cuuint32_t)KS, (cuuint32_t)TM};
        int rc = make_map(&mx, BF, x, 2, dims, row_stride, box, true);
        if (!rc) rc = make_map(&mout, BF, out, 2, dims, row_stride, box, true);
        if (!rc) rc = make_map(&mbase, BF, base ? base : x, 2, dims, row_stride, box, true);
        if (rc) return rc;
    }
    {  // A (E, C, R) as (8 values, C, R / 8 pieces, E): one box is a 64-channel Acat slice
        // in MN-major core matrices (8 channels x 16 bytes), N group e * R / 8 + piece
        const cuuint64_t dims[4] = {8, (cuuint64_t)C, (cuuint64_t)rp, (cuuint64_t)E};
        const cuuint64_t strides[3] = {(cuuint64_t)R * 2, 16, (cuuint64_t)C * R * 2};
        const cuuint32_t box[4] = {8, (cuuint32_t)KS, (cuuint32_t)rp, (cuuint32_t)E};
        const int rc = make_map(&ma, BF, A, 4, dims, strides, box, false);
        if (rc) return rc;
    }
    {  // B (E, R, C) = Bcat (EN, C): box 64 channels x EN rows, 128-byte swizzle
        const cuuint64_t dims[2] = {(cuuint64_t)C, (cuuint64_t)EN};
        const cuuint32_t box[2] = {(cuuint32_t)NC, (cuuint32_t)EN};
        const int rc = make_map(&mb, BF, B, 2, dims, row_stride, box, true);
        if (rc) return rc;
    }
    auto kern = moe_lora_apply_tc_kernel<T, EN, RT>;
    const int smem = Geo<EN, RT>::SMEM;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return set_cuda_error(err);
    const int grid = moe_apply_tc_grid(ntok);
    const int accum = base != nullptr && base == out;
    kern<<<grid, NTH, smem, st>>>(mx, ma, mb, mbase, mout, base ? 1 : 0, accum, inds, (const T*)scores, ntok, C, R,
                                  topk, ra);
    return check_launch();
}

template <typename T>
int moe_lora_apply_tc(const void* x, const void* base, const void* A, const void* B, const int32_t* inds,
                      const void* scores, void* out, int ntok, int C, int R, int E, int topk, cudaStream_t st) {
    const RouteArgs ra{};
    switch (E * R) {
        case 32: return launch_apply_tc<T, 32, false>(x, base, A, B, inds, scores, out, ntok, C, R, topk, ra, st);
        case 64: return launch_apply_tc<T, 64, false>(x, base, A, B, inds, scores, out, ntok, C, R, topk, ra, st);
        case 128: return launch_apply_tc<T, 128, false>(x, base, A, B, inds, scores, out, ntok, C, R, topk, ra, st);
        default: return RWKV_ERR_SHAPE;
    }
}

// Routed variant (fp16): the gate split into `gsplit` (C / 64 blocks of 4 KB), then the
// apply kernel with the router folded into its down product; the per-CTA routing
// partials go to part_f / part_c (moe_apply_tc_grid(ntok) CTAs) for the finalize kernel.
int moe_lora_apply_tc_routed(const void* x, const void* base, const void* A, const void* B, const float* gate_w,
                             const float* bias, int32_t* inds, void* scores, void* gsplit, float* part_f,
                             int32_t* part_c, void* out, int ntok, int C, int R, int E, int topk, cudaStream_t st) {
    const int n = C * atc::GATE_COLS;
    moe_gate_split_kernel<<<(n + 255) / 256, 256, 0, st>>>(gate_w, (__half*)gsplit, E, C);
    int rc = check_launch();
    if (rc) return rc;
    const RouteArgs ra{(const unsigned char*)gsplit, bias, E, inds, scores, part_f, part_c};
    switch (E * R) {
        case 32: return launch_apply_tc<__half, 32, true>(x, base, A, B, nullptr, nullptr, out, ntok, C, R, topk, ra, st);
        case 64: return launch_apply_tc<__half, 64, true>(x, base, A, B, nullptr, nullptr, out, ntok, C, R, topk, ra, st);
        case 128: return launch_apply_tc<__half, 128, true>(x, base, A, B, nullptr, nullptr, out, ntok, C, R, topk, ra, st);
        default: return RWKV_ERR_SHAPE;
    }
}
template int moe_lora_apply_tc<__half>(const void*, const void*, const void*, const void*, const int32_t*,
                                       const void*, void*, int, int, int, int, int, cudaStream_t);
template int moe_lora_apply_tc<__nv_bfloat16>(const void*, const void*, const void*, const void*,
                                              const int32_t*, const void*, void*, int, int, int, int, int,
                                              cudaStream_t);

int read_device_error_moe(int clear) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_error_moe, sizeof(int));
    if (e != cudaSuccess) return -set_cuda_error(e);
    if (clear && v) {
        const int z = 0;
        e = cudaMemcpyToSymbol(g_device_error_moe, &z, sizeof(int));
        if (e != cudaSuccess) return -set_cuda_error(e);
    }
    return v;
}

}  // namespace rwkv

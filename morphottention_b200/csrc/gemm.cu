// gemm.cu -- one warp-specialised tcgen05 GEMM kernel (128 x BN tiles, K blocks of 64,
// TMA-fed multi-stage shared-memory ring, fp32 accumulator in TMEM) with three
// epilogues:
//   * EpiProj  : X @ [W_phi | W_V]   -> sigmoid, gating, bias sums, fp16 codes and V
//                (query codes centered: gate_q * (phi - 1/2), see ProjOut)
//                (replaces the per-tile re-projection of project.cuh:16-47 and
//                attention.cu:102-111, which the reference repeats for every Q block)
//   * EpiHalf  : dcat @ [W_phi | W_V]^T -> dX fp16  (replaces the fp16 atomics of
//                attention.cu:393-402, :462-468 and project.cuh:99)
//   * EpiF32   : X^T @ dcat -> fp32 split-K partials of [dW_phi | dW_V]  (replaces the
//                fp16 atomics of attention.cu:382-390 and project.cuh:89-96)
//
// Warp roles (320 threads): warp 0 = TMA producer, warp 1 = TMEM owner + MMA issuer,
// warps 2-9 = epilogue (warp w reads TMEM lanes 32*(w%4) .. +31, one output row per
// thread; warps 2-5 and 6-9 take the two column halves of a tile when BN >= 128).  Operands are fp16 with 128-byte swizzle; A and B may each be K-major or
// MN-major, which the instruction descriptor's transpose bits express, so no operand
// is ever transposed in memory.
//
// Persistent: one CTA per SM walks the work items (tile, K split) with a stride of the
// grid size; the fp32 accumulator is double-buffered in TMEM (2 x BN columns), so the
// epilogue of one tile overlaps the main loop of the next.  Items are numbered with the
// N tile fastest, so CTAs running at the same time share an A row block in L2.  BN = 256
// where the shape allows: each MMA then does twice the work of an N = 128 one for the
// same per-instruction and per-barrier-probe costs of the issuing thread.
#include "kernels.h"
#include "sm100.cuh"

namespace morpho {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kGemmThreads = 320;  // producer, MMA, 8 epilogue warps

enum BMode : int { B_SINGLE = 0, B_SPLIT_N = 1, B_SPLIT_K = 2 };

// Epilogue staging: per epilogue warp 32 rows of its widest store (Epi::kStageBytes: 4 KB for
// 128-byte fp32 rows, 2 KB for the fp16 dX rows), through which each warp turns its row-per-lane
// results into coalesced global stores (store_rows32).  The dX GEMM keeps its footprint small so
// that the data-parallel all-reduce kernel, which runs beside it, still finds room on its SMs.
template <int BN, int EPI_STAGE>
struct GemmCfg {
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = (196608 / STAGE_BYTES) > 8 ? 8 : (196608 / STAGE_BYTES);  // <= 192 KB of ring
    static constexpr int BAR_OFFSET = STAGES * STAGE_BYTES;
    static constexpr int EPI_OFFSET = BAR_OFFSET + 256;
    // ring + barriers + 8 epilogue staging buffers + 1 KB alignment slack
    static constexpr int SMEM_BYTES = EPI_OFFSET + 8 * EPI_STAGE + 1024;
    static_assert(SMEM_BYTES <= 232448, "smem budget");
    static constexpr uint32_t TMEM_COLS = 2 * BN;                 // double-buffered accumulator
    static_assert(TMEM_COLS <= 512, "TMEM");
};

struct GemmArgs {
    int M, N;
    int k_blocks;      // ceil(K / BK)
    int kb_per_split;  // K blocks handled by one split
    int b_split;       // B_SPLIT_N: first column of B1; B_SPLIT_K: first K index of B1
    int tiles_m, tiles_n, splits;
    uint32_t* status;
};

// ---- epilogues ----------------------------------------------------------------------

template <int NC>
__device__ __forceinline__ void tmem_load_cols(uint32_t taddr, float* out) {
    static_assert(NC % 16 == 0, "columns in multiples of 16");
    uint32_t r[NC];
#pragma unroll
    for (int c = 0; c < NC; c += 16) tmem_ld16(taddr + c, r + c);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < NC; ++i) out[i] = u2f(r[i]);
}

// phi = proj(z) in place (reference morfology/cube.cuh:12-26); the choice is uniform, so
// each branch is one unrolled loop.
template <int NC>
__device__ __forceinline__ void cube_project(float* z, int proj) {
    if (proj == kProjSigmoid) {
#pragma unroll
        for (int i = 0; i < NC; ++i) z[i] = __fdividef(1.0f, 1.0f + __expf(-z[i]));
    } else if (proj == kProjHardTanh01) {
#pragma unroll
        for (int i = 0; i < NC; ++i) z[i] = fminf(1.0f, fmaxf(0.0f, 0.5f * (z[i] + 1.0f)));
    }
}

struct ProjParams {
    int T, N, Npad, H, hd, Hp, D;
    int proj;  // kProj*
    float c;  // scale * log2(e)
    const __half* gq;
    const __half* gk;
    ProjOut o;
};

// Projection epilogue for cube width MC.  Tile columns [n0, n0+BN) of the padded
// output space [0, Hp) -> heads' z values, [Hp, Hp + D) -> V columns.
template <int MC>
struct EpiProj {
    using Params = ProjParams;
    static constexpr int kStageBytes = 4096;  // phi rows: 32 fp32
    template <int BN>
    __device__ static void run(const Params& p, uint32_t tacc, int row, int n0, int /*z*/, uint32_t stage, int lane) {
        const bool live = row < p.T;
        const int b = live ? row / p.N : 0;
        const int n = live ? row - b * p.N : 0;
        // the warp's 32 rows are consecutive tokens of one sequence: coalesced stores through the
        // staging buffer (warp-uniform), else each lane stores its own row
        const int r0 = row - lane;
        const bool coal = r0 + 31 < p.T && r0 / p.N == (r0 + 31) / p.N;
        if (n0 < p.Hp) {
#pragma unroll 1
            for (int hc = 0; hc < BN / MC; ++hc) {
                const int h = n0 / MC + hc;
                if (h >= p.H) break;  // pad columns of the last phi tile
                // the head's MC columns in chunks of CW (bias sums carry over), so that a 64-wide
                // head does not hold all its columns in registers at once
                constexpr int CW = MC < 32 ? MC : 32;
                const __half2* gq2 = reinterpret_cast<const __half2*>(p.gq + h * MC);
                const __half2* gk2 = reinterpret_cast<const __half2*>(p.gk + h * MC);
                const size_t base = static_cast<size_t>(b * p.H + h) * p.N + n;
                float qb = 0.f, cb = 0.f;
#pragma unroll
                for (int q = 0; q < MC / CW; ++q) {
                    float zr[CW];
                    tmem_load_cols<CW>(tacc + hc * MC + q * CW, zr);
                    cube_project<CW>(zr, p.proj);  // zr = phi from here on
                    uint32_t qpk[CW / 2], kpk[CW / 2], hpk[CW / 2], lpk[CW / 2];
#pragma unroll
                    for (int c = 0; c < CW; c += 2) {
                        const float2 gq = __half22float2(gq2[(q * CW + c) / 2]);
                        const float2 gk = __half22float2(gk2[(q * CW + c) / 2]);
                        const float p0 = zr[c];
                        const float p1 = zr[c + 1];
                        const float q0 = gq.x * p0, q1 = gq.y * p1;
                        const float k0 = gk.x * p0, k1 = gk.y * p1;
                        qb = fmaf(gk.x, q0, fmaf(gk.y, q1, qb));
                        cb = fmaf(gq.x, k0, fmaf(gq.y, k1, cb));
                        qpk[c / 2] = pack_half2(q0 - 0.5f * gq.x, q1 - 0.5f * gq.y);  // centered query code
                        kpk[c / 2] = pack_half2(k0, k1);
                        const float c0 = k0 - 0.5f * gk.x, c1 = k1 - 0.5f * gk.y;  // centered key code
                        const __half2 hi = __floats2half2_rn(c0, c1);
                        const float2 hf = __half22float2(hi);
                        hpk[c / 2] = *reinterpret_cast<const uint32_t*>(&hi);
                        lpk[c / 2] = pack_half2(c0 - hf.x, c1 - hf.y);
                    }
                    if (coal) {
                        const size_t b0 = base - lane;
                        auto u4 = [](const uint32_t* a, int g) { return make_uint4(a[4 * g], a[4 * g + 1], a[4 * g + 2], a[4 * g + 3]); };
                        store_rows32<CW * 2>(stage, lane, [&](int g) { return u4(qpk, g); },
                                             reinterpret_cast<uint8_t*>(p.o.qc + b0 * MC + q * CW), MC * 2);
                        store_rows32<CW * 2>(stage, lane, [&](int g) { return u4(kpk, g); },
                                             reinterpret_cast<uint8_t*>(p.o.kc + b0 * MC + q * CW), MC * 2);
                        if (p.o.kdq != nullptr) {
                            store_rows32<CW * 2>(stage, lane, [&](int g) { return u4(hpk, g); },
                                                 reinterpret_cast<uint8_t*>(p.o.kdq + b0 * (2 * MC) + q * CW), MC * 4);
                            store_rows32<CW * 2>(stage, lane, [&](int g) { return u4(lpk, g); },
                                                 reinterpret_cast<uint8_t*>(p.o.kdq + b0 * (2 * MC) + MC + q * CW),
                                                 MC * 4);
                        }
                        if (p.o.phi != nullptr)
                            store_rows32<CW * 4>(stage, lane,
                                                 [&](int g) {
                                                     return make_uint4(__float_as_uint(zr[4 * g]), __float_as_uint(zr[4 * g + 1]),
                                                                       __float_as_uint(zr[4 * g + 2]), __float_as_uint(zr[4 * g + 3]));
                                                 },
                                                 reinterpret_cast<uint8_t*>(p.o.phi + b0 * MC + q * CW), MC * 4);
                    } else if (live) {
                        uint4* dq = reinterpret_cast<uint4*>(p.o.qc + base * MC + q * CW);
                        uint4* dk = reinterpret_cast<uint4*>(p.o.kc + base * MC + q * CW);
#pragma unroll
                        for (int i = 0; i < CW / 8; ++i) {
                            dq[i] = make_uint4(qpk[4 * i], qpk[4 * i + 1], qpk[4 * i + 2], qpk[4 * i + 3]);
                            dk[i] = make_uint4(kpk[4 * i], kpk[4 * i + 1], kpk[4 * i + 2], kpk[4 * i + 3]);
                        }
                        if (p.o.kdq != nullptr) {
                            uint4* dh = reinterpret_cast<uint4*>(p.o.kdq + base * (2 * MC) + q * CW);
                            uint4* dl = reinterpret_cast<uint4*>(p.o.kdq + base * (2 * MC) + MC + q * CW);
#pragma unroll
                            for (int i = 0; i < CW / 8; ++i) {
                                dh[i] = make_uint4(hpk[4 * i], hpk[4 * i + 1], hpk[4 * i + 2], hpk[4 * i + 3]);
                                dl[i] = make_uint4(lpk[4 * i], lpk[4 * i + 1], lpk[4 * i + 2], lpk[4 * i + 3]);
                            }
                        }
                        if (p.o.phi != nullptr) {
                            float4* dp = reinterpret_cast<float4*>(p.o.phi + base * MC + q * CW);
#pragma unroll
                            for (int i = 0; i < CW / 4; ++i)
                                dp[i] = make_float4(zr[4 * i], zr[4 * i + 1], zr[4 * i + 2], zr[4 * i + 3]);
                        }
                    }
                }
                if (live) {
                    const size_t brow = static_cast<size_t>(b * p.H + h) * p.Npad + n;  // padded bias rows
                    p.o.qb[brow] = qb * p.c;
                    p.o.cb[brow] = cb * p.c;
                }
            }
        } else {
            // the next 32-column chunk's TMEM load is in flight while this one is stored
            uint32_t rb[2][32];
            tmem_ld32(tacc, rb[0]);
            tmem_ld_wait();
#pragma unroll
            for (int cc = 0; cc < BN / 32; ++cc) {
                const int g = n0 - p.Hp + cc * 32;  // V column
                if (g >= p.D) break;
                const uint32_t* r = rb[cc & 1];
                if (cc + 1 < BN / 32 && g + 32 < p.D) tmem_ld32(tacc + (cc + 1) * 32, rb[(cc + 1) & 1]);
                if (coal) {
                    const int h = g / p.hd;
                    const int e = g - h * p.hd;
                    const size_t b0 = static_cast<size_t>(b * p.H + h) * p.N + n - lane;
                    store_rows32<64>(stage, lane,
                                     [&](int i) {
                                         return make_uint4(pack_half2(u2f(r[8 * i]), u2f(r[8 * i + 1])),
                                                           pack_half2(u2f(r[8 * i + 2]), u2f(r[8 * i + 3])),
                                                           pack_half2(u2f(r[8 * i + 4]), u2f(r[8 * i + 5])),
                                                           pack_half2(u2f(r[8 * i + 6]), u2f(r[8 * i + 7])));
                                     },
                                     reinterpret_cast<uint8_t*>(p.o.v + b0 * p.hd + e), static_cast<size_t>(p.hd) * 2);
                } else if (live) {
                    const int h = g / p.hd;
                    const int e = g - h * p.hd;
                    uint4* dv = reinterpret_cast<uint4*>(p.o.v + (static_cast<size_t>(b * p.H + h) * p.N + n) * p.hd + e);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        dv[i] = make_uint4(pack_half2(u2f(r[8 * i]), u2f(r[8 * i + 1])),
                                           pack_half2(u2f(r[8 * i + 2]), u2f(r[8 * i + 3])),
                                           pack_half2(u2f(r[8 * i + 4]), u2f(r[8 * i + 5])),
                                           pack_half2(u2f(r[8 * i + 6]), u2f(r[8 * i + 7])));
                }
                tmem_ld_wait();
            }
        }
    }
};

struct HalfParams {
    int M, N, ld;
    __half* out;
};

struct EpiHalf {
    using Params = HalfParams;
    static constexpr int kStageBytes = 2048;  // 32 fp16 columns
    template <int BN>
    __device__ static void run(const Params& p, uint32_t tacc, int row, int n0, int /*z*/, uint32_t stage, int lane) {
        const bool coal = row - lane + 31 < p.M;  // warp-uniform: all 32 rows exist
        // the next 32-column chunk's TMEM load is in flight while this one is stored
        uint32_t rb[2][32];
        tmem_ld32(tacc, rb[0]);
        tmem_ld_wait();
#pragma unroll
        for (int cc = 0; cc < BN / 32; ++cc) {
            const int col = n0 + cc * 32;
            if (col >= p.N) break;
            const uint32_t* r = rb[cc & 1];
            if (cc + 1 < BN / 32 && col + 32 < p.N) tmem_ld32(tacc + (cc + 1) * 32, rb[(cc + 1) & 1]);
            if (coal) {
                store_rows32<64>(stage, lane,
                                 [&](int i) {
                                     return make_uint4(pack_half2(u2f(r[8 * i]), u2f(r[8 * i + 1])),
                                                       pack_half2(u2f(r[8 * i + 2]), u2f(r[8 * i + 3])),
                                                       pack_half2(u2f(r[8 * i + 4]), u2f(r[8 * i + 5])),
                                                       pack_half2(u2f(r[8 * i + 6]), u2f(r[8 * i + 7])));
                                 },
                                 reinterpret_cast<uint8_t*>(p.out + static_cast<size_t>(row - lane) * p.ld + col),
                                 static_cast<size_t>(p.ld) * 2);
            } else if (row < p.M) {
                uint4* dst = reinterpret_cast<uint4*>(p.out + static_cast<size_t>(row) * p.ld + col);
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    dst[i] = make_uint4(pack_half2(u2f(r[8 * i]), u2f(r[8 * i + 1])),
                                        pack_half2(u2f(r[8 * i + 2]), u2f(r[8 * i + 3])),
                                        pack_half2(u2f(r[8 * i + 4]), u2f(r[8 * i + 5])),
                                        pack_half2(u2f(r[8 * i + 6]), u2f(r[8 * i + 7])));
            }
            tmem_ld_wait();
        }
    }
};

struct F32Params {
    int M, N, ld;
    float* out;  // [splits, M, ld]
};

struct EpiF32 {
    using Params = F32Params;
    static constexpr int kStageBytes = 4096;  // 32 fp32 columns
    template <int BN>
    __device__ static void run(const Params& p, uint32_t tacc, int row, int n0, int z, uint32_t stage, int lane) {
        const bool coal = row - lane + 31 < p.M;  // warp-uniform: all 32 rows exist
        // the next 32-column chunk's TMEM load is in flight while this one is stored
        uint32_t rb[2][32];
        tmem_ld32(tacc, rb[0]);
        tmem_ld_wait();
#pragma unroll
        for (int cc = 0; cc < BN / 32; ++cc) {
            const int col = n0 + cc * 32;
            if (col >= p.N) break;
            const uint32_t* r = rb[cc & 1];
            if (cc + 1 < BN / 32 && col + 32 < p.N) tmem_ld32(tacc + (cc + 1) * 32, rb[(cc + 1) & 1]);
            if (coal) {
                store_rows32<128>(stage, lane,
                                  [&](int i) { return make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]); },
                                  reinterpret_cast<uint8_t*>(p.out + (static_cast<size_t>(z) * p.M + row - lane) * p.ld + col),
                                  static_cast<size_t>(p.ld) * 4);
            } else if (row < p.M) {
                float4* dst = reinterpret_cast<float4*>(p.out + (static_cast<size_t>(z) * p.M + row) * p.ld + col);
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    dst[i] = make_float4(u2f(r[4 * i]), u2f(r[4 * i + 1]), u2f(r[4 * i + 2]), u2f(r[4 * i + 3]));
            }
            tmem_ld_wait();
        }
    }
};

// ---- the kernel ---------------------------------------------------------------------

// A is M x K, B is K x N (logical).  A_MN: A stored [K, M] (M contiguous), else [M, K].
// B_MN: B stored [K, N] (N contiguous), else [N, K].
template <int BN, bool A_MN, bool B_MN, int BMODE, class Epi>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
                const __grid_constant__ CUtensorMap tmB1, const GemmArgs args, const typename Epi::Params ep) {
    using Cfg = GemmCfg<BN, Epi::kStageBytes>;
    constexpr int STAGES = Cfg::STAGES;
    // epilogue warps 2..9; with BN >= 128 each of the two warpgroups takes half the columns,
    // with BN = 64 only warps 2..5 work
    constexpr int kEpiGroups = BN >= 128 ? 2 : 1;
    constexpr int kEpiWarps = 4 * kEpiGroups;
    constexpr int kEpiCols = BN / kEpiGroups;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::BAR_OFFSET);
    // bars[0..S) full, bars[S..2S) empty, then acc_full[2], acc_empty[2], drain
    constexpr int NB = 2 * STAGES + 5;
    static_assert(NB * 8 + 8 <= 256, "barrier block");
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NB);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const int warp = warp_id();
    const int lane = threadIdx.x & 31;
    const int n_items = args.tiles_m * args.tiles_n * args.splits;
    const int mn_tiles = args.tiles_m * args.tiles_n;
    // work item -> (m0, n0, split): N tile fastest, then M tile, then split
    auto decode = [&](int w, int& m0, int& n0, int& z) {
        z = w / mn_tiles;
        const int r = w - z * mn_tiles;
        const int mt = r / args.tiles_n;
        m0 = mt * BM;
        n0 = (r - mt * args.tiles_n) * BN;
    };

    const uint32_t full0 = smem_u32(bars);
    const uint32_t empty0 = smem_u32(bars + STAGES);
    const uint32_t acc_full0 = smem_u32(bars + 2 * STAGES);      // + 8 * buffer
    const uint32_t acc_empty0 = smem_u32(bars + 2 * STAGES + 2);  // + 8 * buffer
    const uint32_t drain_bar = smem_u32(bars + 2 * STAGES + 4);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(acc_full0 + 8 * a, 1);
            mbar_init(acc_empty0 + 8 * a, kEpiWarps);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0u;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB0);
        if (BMODE != B_SINGLE) tma_prefetch_desc(&tmB1);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), Cfg::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int g = 0;  // K blocks loaded so far, over all items: ring slot and phase
            for (int w = blockIdx.x; w < n_items && !*abort_flag; w += gridDim.x) {
                int m0, n0, z;
                decode(w, m0, n0, z);
                const int kb0 = z * args.kb_per_split;
                const int kb1 = min(args.k_blocks, kb0 + args.kb_per_split);
                for (int kb = kb0; kb < kb1; ++kb, ++g) {
                    const int s = g % STAGES;
                    if (g >= STAGES && !mbar_wait(empty0 + 8 * s, ((g / STAGES) & 1) ^ 1, args.status, K_GEMM, 1)) {
                        *abort_flag = 1u;
                        break;
                    }
                    const uint32_t sA = smem_u32(smem + s * Cfg::STAGE_BYTES);
                    const uint32_t sB = sA + Cfg::A_BYTES;
                    const uint32_t fb = full0 + 8 * s;
                    const int k0 = kb * BK;
                    mbar_arrive_expect_tx(fb, Cfg::STAGE_BYTES);
                    if (A_MN) {
                        tma_load_2d(sA, &tmA, fb, m0, k0);
                        tma_load_2d(sA + 64 * 128, &tmA, fb, m0 + 64, k0);
                    } else {
                        tma_load_2d(sA, &tmA, fb, k0, m0);
                    }
                    const CUtensorMap* tb = &tmB0;
                    int bn = n0, bk = k0;
                    if (BMODE == B_SPLIT_N && n0 >= args.b_split) {
                        tb = &tmB1;
                        bn = n0 - args.b_split;
                    }
                    if (BMODE == B_SPLIT_K && k0 >= args.b_split) {
                        tb = &tmB1;
                        bk = k0 - args.b_split;
                    }
                    if (B_MN) {
#pragma unroll
                        for (int c = 0; c < BN / 64; ++c) tma_load_2d(sB + c * 64 * 128, tb, fb, bn + 64 * c, bk);
                    } else {
                        tma_load_2d(sB, tb, fb, bk, bn);
                    }
                }
            }
            // Drain: wait (bounded) for this thread's loads still in flight.
            if (*abort_flag) {
                for (int i = max(0, g - STAGES); i < g; ++i)
                    mbar_wait(full0 + 8 * (i % STAGES), (i / STAGES) & 1, args.status, K_GEMM, 2);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        // The whole warp runs this loop (warp-uniform control flow and descriptor arithmetic);
        // elect.sync inside umma_ss_w / umma_commit_w lets one lane issue each instruction, so the
        // issuer is not a divergent lane beside the epilogue warps of its sub-partition.
        {
            constexpr uint32_t idesc = make_idesc_f16(BM, BN, A_MN, B_MN);
            bool ok = true;
            int g = 0;  // K blocks consumed so far
            int j = 0;  // items of this CTA so far: accumulator buffer j & 1
            for (int w = blockIdx.x; ok && w < n_items; w += gridDim.x, ++j) {
                int m0, n0, z;
                decode(w, m0, n0, z);
                const int kb0 = z * args.kb_per_split;
                const int nkb = min(args.k_blocks, kb0 + args.kb_per_split) - kb0;
                const int a = j & 1;
                // the epilogue warps have drained this buffer (its previous use, item j - 2)
                if (j >= 2 && !mbar_wait_warp(acc_empty0 + 8 * a, ((j >> 1) & 1) ^ 1, args.status, K_GEMM, 6)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t dacc = tmem + a * BN;
                for (int i = 0; i < nkb; ++i, ++g) {
                    const int s = g % STAGES;
                    if (!mbar_wait_warp(full0 + 8 * s, (g / STAGES) & 1, args.status, K_GEMM, 3)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sA = smem_u32(smem + s * Cfg::STAGE_BYTES);
                    const uint32_t sB = sA + Cfg::A_BYTES;
#pragma unroll
                    for (int ks = 0; ks < BK / 16; ++ks) {
                        const uint64_t ad = A_MN ? make_sdesc(sA + ks * 2048, 64 * 128, 1024, SW_128)
                                                 : make_sdesc(sA + ks * 32, 16, 1024, SW_128);
                        const uint64_t bd = B_MN ? make_sdesc(sB + ks * 2048, 64 * 128, 1024, SW_128)
                                                 : make_sdesc(sB + ks * 32, 16, 1024, SW_128);
                        umma_ss_w(dacc, ad, bd, idesc, (i > 0 || ks > 0) ? 1u : 0u);
                    }
                    umma_commit_w(empty0 + 8 * s);
                }
                if (ok) umma_commit_w(acc_full0 + 8 * a);
            }
            if (!ok) {
                *abort_flag = 1u;
                umma_commit_w(drain_bar);
                mbar_wait_warp(drain_bar, 0, args.status, K_GEMM, 4);
                // release the epilogue warps' next wait on either buffer
                umma_commit_w(acc_full0);
                umma_commit_w(acc_full0 + 8);
            }
        }
    } else if (warp - 2 < kEpiWarps) {
        // ---------------- epilogue (warps 2..9) ----------------
        const int quad = warp & 3;
        const int half = (warp - 2) >> 2;  // column half of the tile
        const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
        const uint32_t estage = smem_u32(smem + Cfg::EPI_OFFSET + (warp - 2) * Epi::kStageBytes);
        int j = 0;
        for (int w = blockIdx.x; w < n_items; w += gridDim.x, ++j) {
            int m0, n0, z;
            decode(w, m0, n0, z);
            const int a = j & 1;
            if (!mbar_wait_warp(acc_full0 + 8 * a, (j >> 1) & 1, args.status, K_GEMM, 5) || *abort_flag) {
                *abort_flag = 1u;
                break;
            }
            tc_fence_after();
            Epi::template run<kEpiCols>(ep, tmem + a * BN + half * kEpiCols + lane_off, m0 + quad * 32 + lane,
                                        n0 + half * kEpiCols, z, estage, lane);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty0 + 8 * a);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::TMEM_COLS);
    }
}

template <int BN, bool A_MN, bool B_MN, int BMODE, class Epi>
int run_gemm(const CUtensorMap& tmA, const CUtensorMap& tmB0, const CUtensorMap& tmB1, const GemmArgs& args,
             const typename Epi::Params& ep, int splits, int sms, cudaStream_t stream, const char* name) {
    auto kern = gemm_kernel<BN, A_MN, B_MN, BMODE, Epi>;
    constexpr int smem = GemmCfg<BN, Epi::kStageBytes>::SMEM_BYTES;
    MORPHO_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    GemmArgs a = args;
    a.tiles_m = (args.M + BM - 1) / BM;
    a.tiles_n = (args.N + BN - 1) / BN;
    a.splits = splits;
    const int items = a.tiles_m * a.tiles_n * splits;
    // Persistent CTAs, at most one per SM, dealt the items round-robin: as few CTAs as keep the
    // largest per-CTA count (the kernel's length) leaves the other SMs free for concurrent work,
    // e.g. the data-parallel all-reduce beside the dX GEMM (c3: 512 tiles on 128 of 148 SMs).
    const int per_cta = (items + sms - 1) / sms;
    const int grid = (items + per_cta - 1) / per_cta;
    prof_begin(stream, name);
    kern<<<grid, kGemmThreads, smem, stream>>>(tmA, tmB0, tmB1, a, ep);
    MORPHO_LAUNCH_CHECK(name);
    return MORPHO_OK;
}

}  // namespace

// ---- launchers ----------------------------------------------------------------------

int launch_proj(const DeviceInfo& dev, const Shape& s, const __half* X, const __half* W_phi, const __half* W_V,
                const __half* gate_q, const __half* gate_k, const ProjOut& o, cudaStream_t stream) {
    const long long T = s.tokens();
    const int Hp = s.Hp();
    // tiles never straddle the phi / V column boundary Hp
    const int BN = (Hp % 256 == 0 && s.D % 256 == 0) ? 256 : (Hp % 128 == 0 && s.D % 128 == 0) ? 128 : 64;
    CUtensorMap tA, tB0, tB1;
    MORPHO_TRY(make_tmap_2d_f16(&tA, X, T, s.D, s.D, BM, BK));
    MORPHO_TRY(make_tmap_2d_f16(&tB0, W_phi, s.D, s.Hm(), s.Hm(), BK, 64));
    MORPHO_TRY(make_tmap_2d_f16(&tB1, W_V, s.D, s.D, s.D, BK, 64));
    GemmArgs a;
    a.M = static_cast<int>(T);
    a.N = s.Cp();
    a.k_blocks = (s.D + BK - 1) / BK;
    a.kb_per_split = a.k_blocks;
    a.b_split = Hp;
    a.status = dev.status;
    ProjParams p;
    p.T = static_cast<int>(T);
    p.N = s.N;
    p.Npad = (s.N + 127) / 128 * 128;
    p.H = s.H;
    p.hd = s.hd;
    p.Hp = Hp;
    p.D = s.D;
    p.c = s.scale * kLog2e;
    p.proj = s.proj;
    p.gq = gate_q;
    p.gk = gate_k;
    p.o = o;
    switch (s.m) {
        case 16:
            return BN == 256   ? run_gemm<256, false, true, B_SPLIT_N, EpiProj<16>>(tA, tB0, tB1, a, p, 1, dev.sms, stream, "proj")
                   : BN == 128 ? run_gemm<128, false, true, B_SPLIT_N, EpiProj<16>>(tA, tB0, tB1, a, p, 1, dev.sms, stream, "proj")
                               : run_gemm<64, false, true, B_SPLIT_N, EpiProj<16>>(tA, tB0, tB1, a, p, 1, dev.sms, stream, "proj");
        case 32:
            return BN == 256   ? run_gemm<256, false, true, B_SPLIT_N, EpiProj<32>>(tA, tB0, tB1, a, p, 1, dev.sms, stream, "proj")
                   : BN == 128 ? run_gemm<128, false, true, B_SPLIT_N, EpiProj<32>>(tA, tB0, tB1, a, p, 1, dev.sms, stream, "proj")
                               : run_gemm<64, false, true, B_SPLIT_N, EpiProj<32>>(tA, tB0, tB1, a, p, 1, dev.sms, stream, "proj");
        case 64:
            return BN == 256   ? run_gemm<256, false, true, B_SPLIT_N, EpiProj<64>>(tA, tB0, tB1, a, p, 1, dev.sms, stream, "proj")
                   : BN == 128 ? run_gemm<128, false, true, B_SPLIT_N, EpiProj<64>>(tA, tB0, tB1, a, p, 1, dev.sms, stream, "proj")
                               : run_gemm<64, false, true, B_SPLIT_N, EpiProj<64>>(tA, tB0, tB1, a, p, 1, dev.sms, stream, "proj");
        default:
            return set_error(MORPHO_ERR_INVALID, "cube_m %d not supported (16, 32 or 64)", s.m);
    }
}

int launch_dx(const DeviceInfo& dev, const Shape& s, const __half* dcat, const __half* W_phi, const __half* W_V,
              __half* dX, cudaStream_t stream) {
    const long long T = s.tokens();
    const int BN = s.D % 256 == 0 ? 256 : 128;
    CUtensorMap tA, tB0, tB1;
    MORPHO_TRY(make_tmap_2d_f16(&tA, dcat, T, s.Cp(), s.Cp(), BM, BK));
    // B^T = [W_phi | W_V] viewed as K-major [D rows, K cols]
    MORPHO_TRY(make_tmap_2d_f16(&tB0, W_phi, s.D, s.Hm(), s.Hm(), BN, BK));
    MORPHO_TRY(make_tmap_2d_f16(&tB1, W_V, s.D, s.D, s.D, BN, BK));
    GemmArgs a;
    a.M = static_cast<int>(T);
    a.N = s.D;
    a.k_blocks = (s.Cp() + BK - 1) / BK;
    a.kb_per_split = a.k_blocks;
    a.b_split = s.Hp();
    a.status = dev.status;
    HalfParams p;
    p.M = a.M;
    p.N = s.D;
    p.ld = s.D;
    p.out = dX;
    return BN == 256 ? run_gemm<256, false, false, B_SPLIT_K, EpiHalf>(tA, tB0, tB1, a, p, 1, dev.sms, stream, "dx_gemm")
                     : run_gemm<128, false, false, B_SPLIT_K, EpiHalf>(tA, tB0, tB1, a, p, 1, dev.sms, stream, "dx_gemm");
}

// N tile of the dW GEMM (its output columns are [0, Cp)).
int dw_bn(const Shape& s) { return s.Cp() % 256 == 0 ? 256 : 128; }

int dw_splits(const DeviceInfo& dev, const Shape& s) {
    const int BN = dw_bn(s);
    const int tiles = ((s.D + BM - 1) / BM) * ((s.Cp() + BN - 1) / BN);
    const int kblocks = static_cast<int>((s.tokens() + BK - 1) / BK);
    // About one work item per SM (persistent CTAs), at least 8 K blocks per split; the
    // split count is then reduced until no split is empty.
    int splits = max(1, min(dev.sms / tiles, kblocks / 8));
    while (splits > 1) {
        const int per = (kblocks + splits - 1) / splits;
        if ((kblocks + per - 1) / per == splits) break;
        --splits;
    }
    return splits;
}

int launch_dw(const DeviceInfo& dev, const Shape& s, const __half* X, const __half* dcat, float* part, int splits,
              cudaStream_t stream) {
    const long long T = s.tokens();
    const int BN = dw_bn(s);
    CUtensorMap tA, tB0;
    // A = X^T: stored [T (K), D (M)] -> MN-major boxes of 64 x 64.
    MORPHO_TRY(make_tmap_2d_f16(&tA, X, T, s.D, s.D, BK, 64));
    // B = dcat: stored [T (K), Cp (N)] -> MN-major boxes of 64 x 64.
    MORPHO_TRY(make_tmap_2d_f16(&tB0, dcat, T, s.Cp(), s.Cp(), BK, 64));
    GemmArgs a;
    a.M = s.D;
    a.N = s.Cp();
    a.k_blocks = static_cast<int>((T + BK - 1) / BK);
    a.kb_per_split = (a.k_blocks + splits - 1) / splits;
    a.b_split = 0;
    a.status = dev.status;
    const int real_splits = (a.k_blocks + a.kb_per_split - 1) / a.kb_per_split;
    if (real_splits != splits)
        return set_error(MORPHO_ERR_INVALID, "internal: dW split count %d does not cover %d K blocks", splits,
                         a.k_blocks);
    F32Params p;
    p.M = s.D;
    p.N = s.Cp();
    p.ld = s.Cp();
    p.out = part;
    return BN == 256 ? run_gemm<256, true, true, B_SINGLE, EpiF32>(tA, tB0, tB0, a, p, splits, dev.sms, stream, "dw_gemm")
                     : run_gemm<128, true, true, B_SINGLE, EpiF32>(tA, tB0, tB0, a, p, splits, dev.sms, stream, "dw_gemm");
}

}  // namespace morpho

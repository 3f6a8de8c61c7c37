// attn_bwd.cu -- MorphoAttention attention backward on sm_100a, KV-stationary.
//
// One CTA = one 128-key tile (kv0 .. kv0+127) of one (batch, head); it loops over the
// query tiles.  TMEM lane j = key row j.  Per query tile i (each product per query half
// h = 0, 1 where it depends on one half, see below):
//   S^T  = Kc . Qc_i^T          (M=128 keys, N=64 queries per half, K=cube_m)  TMEM [0,128)
//       (centered query codes: S = k.q - cb_j/2)
//   dP^T = V . dO_i^T           (K=head_dim, N=64 per half)                  TMEM [P_SEP ? 192 : 128, +128)
//   softmax warps: P^T = 2^(2*scale*log2e*S - cb'_j - L_i), L = lse + qb' (recompute
//       from lse as attention.cu:351-368 does), written back as fp16 into TMEM (own columns
//       where they fit, else over S);
//       dS^T = P^T (dP^T - delta_i) (attention.cu:409-421), fp16 into the dP columns and
//       into a 128B-swizzled shared dS tile; dcb_j += sum_i dS (attention.cu:430-437).
//   dV += P^T . dO_i            (A = P^T from TMEM)                       TMEM [256, +hd)
//   dK += dS^T . Qc_i           (A = dS^T from TMEM, B = Qc MN-major)      TMEM [.., +m)
//       (centered codes: this is dk + gate_q * dcb, whose cancelling bias term is exact)
//   dQ_i = dS . Kc              (A = dS from smem, MN-major)               TMEM [.., +m)
//   dQ warps: dq[b,h,q,:] += 2*scale * dQ_i  (fp32 TMA reduce-add into a workspace: each
//       warp stages its 32 rows in the shared dS tile, free between the dQ MMA and the next
//       dS, and issues one bulk tensor reduce per 32-column box; scattered per-thread global
//       reductions contended with the tensor core's shared-memory operand reads)
// The two softmax warpgroups (query halves h = 0, 1 of each tile) run as two pipelines half a
// tile apart, so that on every SM sub-partition one warpgroup's exponentials overlap the other's
// dS phase: every MMA that depends on one half is issued per half (S_h and dP_h as N = 64, dV_h
// and dK_h as K = 64; dQ whole, once both halves of dS are in shared memory), with per-half
// barriers, by one warp-converged MMA warp in a fixed interleaved order (see the issuer).  Where
// shared memory allows, the dS tile is double-buffered, so neither half waits for the other's dQ.
// Scale factors: dL/dS_raw = 2*scale*dS and dL/dcbias = -scale*sum_i dS (attention.cu:425,
// :436, :442).  Unlike the reference there are no fp16 global atomics: dV and dK are
// complete per CTA and stored once; only dq is accumulated, in fp32.
//
// Warps (512 threads, four warpgroups): warp 0 = TMA producer, warp 1 = TMEM owner + MMA
// issuer (warps 2-3 idle), warps 4..7 softmax for queries [0,64) of the tile (half 0), 8..11
// softmax for queries [64,128) (half 1), 12..15 dQ epilogue.  setmaxnreg moves registers from the producer
// and dQ warpgroups to the two softmax warpgroups.
#include "kernels.h"
#include "sm100.cuh"

namespace morpho {
namespace {

constexpr int kBwdThreads = 512;
constexpr int kTile = 128;
// Register split (512 threads x 128 at launch = 65536): producer/MMA warpgroup 96, dQ
// warpgroup 64, the two softmax warpgroups 176 each; 128*96 + 128*64 + 256*176 = 65536.
constexpr uint32_t kRegsProducer = 96;
constexpr uint32_t kRegsDq = 64;
constexpr uint32_t kRegsSoftmax = 176;
static_assert(128 * kRegsProducer + 128 * kRegsDq + 256 * kRegsSoftmax == 65536, "register split");

template <int MC, int HD>
struct BwdStages {
    // Fixed buffers, then as many query-tile stages (Q, dO, bias slice, L) as fit in the
    // 232448-byte opt-in shared memory, up to 4: the next tiles' loads must be issued well
    // ahead of the MMA that needs them.
    static constexpr int KC = kTile * MC * 2;
    static constexpr int KCS = (KC + 1023) / 1024 * 1024;
    static constexpr int VB = kTile * HD * 2;
    static constexpr int FIXED = 3 * KCS + VB + 2 * kTile * 128 + kTile * 32 + kTile * 4 + 256 + 1024;
    static constexpr int STAGE = KCS + VB + kTile * 32 + kTile * 4;
    // A second dS tile (32 KB) where it fits beside at least two stages: then the two query
    // halves never wait for each other's dQ (see the dQ staging and dq_free below).
    static constexpr int DS2_EXTRA = 2 * kTile * 128;
    static constexpr bool ds2 = FIXED + DS2_EXTRA + 2 * STAGE <= 232448;
    static constexpr int FIX = FIXED + (ds2 ? DS2_EXTRA : 0);
    static constexpr int value = FIX + 4 * STAGE <= 232448 ? 4 : (FIX + 3 * STAGE <= 232448 ? 3 : 2);
};

template <int MC, int HD>
struct BwdCfg {
    static constexpr int kQStages = BwdStages<MC, HD>::value;
    static constexpr bool DS2 = BwdStages<MC, HD>::ds2;  // two dS tiles, alternating per query tile
    static constexpr int N_DS = DS2 ? 2 : 1;
    static constexpr int KC_BYTES = kTile * MC * 2;  // one code tile (K or Q)
    static constexpr int V_BYTES = kTile * HD * 2;   // one V or dO tile
    static constexpr int KC_STRIDE = (KC_BYTES + 1023) / 1024 * 1024;
    // dQ = dS . [hi | lo]: one MMA with N = 2m when its TMEM columns fit (m <= 32), else
    // two accumulating N = m passes.
    static constexpr bool DQ_MERGED = MC <= 32;
    static constexpr int DQ_COLS = DQ_MERGED ? 2 * MC : MC;
    static constexpr uint32_t KD_ROW = DQ_MERGED ? 4 * MC : 128;  // bytes per row of one kdq chunk
    static constexpr int OFF_K = 0;
    static constexpr int OFF_KD = OFF_K + KC_STRIDE;  // centered key codes [hi | lo] (dQ MMA)
    static constexpr int OFF_V = OFF_KD + 2 * KC_STRIDE;
    static constexpr int OFF_Q = OFF_V + V_BYTES;
    static constexpr int OFF_DO = OFF_Q + kQStages * KC_STRIDE;
    static constexpr int OFF_DS = OFF_DO + kQStages * V_BYTES;  // 2 chunks x 128 rows x 128 B
    static constexpr int DS_BYTES = 2 * kTile * 128;
    static constexpr int AUG_BYTES = kTile * 16 * 2;  // one 16-column bias slice
    static constexpr int OFF_VAUG = OFF_DS + N_DS * DS_BYTES;
    static constexpr int OFF_QAUG = OFF_VAUG + AUG_BYTES;
    static constexpr int OFF_L = OFF_QAUG + kQStages * AUG_BYTES;
    static constexpr int OFF_DCB = OFF_L + kQStages * kTile * 4;
    static constexpr int OFF_BAR = OFF_DCB + kTile * 4;
    static constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
    static constexpr int STAGE_TX = KC_BYTES + V_BYTES + AUG_BYTES + kTile * 4;
    // TMEM columns: S 128 | [P 64] | dP 128 | dV hd | dK m | dQ.  When the 64 columns fit,
    // P (fp16) has its own columns, so S_{i+1} can be issued as soon as the softmax warps
    // have read S_i; otherwise P overwrites the first half of each S half and S_{i+1} waits
    // for dV_i.
    static constexpr bool P_SEP = 256 + 64 + HD + MC + DQ_COLS <= 512;
    static constexpr uint32_t TM_S = 0;
    static constexpr uint32_t TM_P = 128;  // used when P_SEP
    static constexpr uint32_t TM_DP = P_SEP ? 192 : 128;
    static constexpr uint32_t TM_DV = TM_DP + 128;
    static constexpr uint32_t TM_DK = TM_DV + HD;
    static constexpr uint32_t TM_DQ = TM_DK + MC;
    // first TMEM column of query half w's P (64 queries as 32 fp16 pairs)
    static constexpr uint32_t p_col(int w) { return P_SEP ? TM_P + 32 * w : TM_S + 64 * w; }
    static constexpr uint32_t TMEM_COLS = 512;
    static_assert(TM_DQ + DQ_COLS <= TMEM_COLS, "TMEM budget (dQ)");
    static constexpr uint32_t KC_ROW = MC * 2;
    static constexpr uint32_t V_ROW = (HD > 64 ? 64 : HD) * 2;

    static_assert(SMEM_BYTES <= 232448, "smem budget");
    static_assert(OFF_DS % 1024 == 0, "the dS tile (also the dQ staging, 128-byte swizzle) is 1024-byte aligned");
};

struct BwdArgs {
    int N, Npad, H, D, Hp, Cp, n_qtiles;
    int BH, band;   // causal launch order (causal_order)
    int mask_diag;  // also drop key j == query i
    float c2;     // 2 * scale * log2(e)
    float two_scale;
    float neg_scale;
    const float* cb;  // [BH, Npad] scaled column bias
    __half* dcat;
    float* dk;   // [BH, N, MC]
    float* dcb;  // [BH, Npad]
    float* dq;   // [BH, N, MC]
    uint32_t* status;
};

// A-operand descriptor for a K-major tile of 128 rows whose K extent may span two
// 64-element chunks (head_dim 128).
template <uint32_t ROW_BYTES>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int ks) {
    constexpr uint32_t sw = swizzle_code_for_row_bytes(ROW_BYTES);
    constexpr int per_chunk = ROW_BYTES / 32;  // K steps of 16 elements per 64-element chunk
    const uint32_t addr = base + (ks / per_chunk) * (kTile * ROW_BYTES) + (ks % per_chunk) * 32;
    return make_sdesc(addr, 16, 8 * ROW_BYTES, sw);
}

template <int MC, int HD, bool CAUSAL, bool SPLIT>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmKD,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                    const __grid_constant__ CUtensorMap tmL, const __grid_constant__ CUtensorMap tmQaug,
                    const __grid_constant__ CUtensorMap tmDQ, const BwdArgs args) {
    using Cfg = BwdCfg<MC, HD>;
    constexpr int kQStages = Cfg::kQStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
    // bars: [0,S) q_full, [S,2S) q_empty, kv_full, then per query half h (two each): s_full,
    //       dp_full, p_full, ds_full, s_free, dv_done; then dq_full, dq_free (one per dS tile),
    //       all_done, drain; TMEM slot and abort flag after them (256 B total)
    constexpr int NB = 2 * kQStages + 18;
    static_assert(NB * 8 + 8 <= 256, "barrier block");
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NB);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const int warp = warp_id();
    const int lane = threadIdx.x & 31;
    int kt, bh;
    if (CAUSAL) {  // key tile kt meets n_qtiles - kt query tiles: heaviest first
        causal_order(static_cast<int>(blockIdx.x), args.n_qtiles, args.BH, args.band, kt, bh);
    } else {
        kt = static_cast<int>(blockIdx.x);
        bh = static_cast<int>(blockIdx.y);
    }
    const int b = bh / args.H;
    const int h = bh - b * args.H;
    const int kv0 = kt * kTile;
    const int i_begin = CAUSAL ? kt : 0;
    const int n_it = args.n_qtiles - i_begin;

    const uint32_t q_full0 = smem_u32(bars);
    const uint32_t q_empty0 = smem_u32(bars + kQStages);
    const uint32_t kv_full = smem_u32(bars + 2 * kQStages);
    // Per query half h (queries 64h .. 64h+63 of a tile, softmax warpgroup h): the two halves run
    // as separate pipelines half a tile apart, so that on every SM sub-partition one warpgroup's
    // exponentials overlap the other's dS phase.
    auto s_full = [&](int h) { return kv_full + 8 * (1 + h); };    // S_h ready
    auto dp_full = [&](int h) { return kv_full + 8 * (3 + h); };   // dP_h ready
    auto p_full = [&](int h) { return kv_full + 8 * (5 + h); };    // P_h in TMEM, dP_h read
    auto ds_full = [&](int h) { return kv_full + 8 * (7 + h); };   // dS_h in TMEM and shared memory
    auto s_free = [&](int h) { return kv_full + 8 * (9 + h); };    // S_h read (and the next stage landed)
    auto dv_done = [&](int h) { return kv_full + 8 * (11 + h); };  // dV_h has read P_h
    const uint32_t dq_full = kv_full + 8 * 13;
    // dq_free(b): the dQ warps have read dQ_i out of TMEM and the TMA has read the rows they staged
    // in dS tile b = i % N_DS, so tile b and the dQ accumulator are free again
    auto dq_free = [&](int b) { return kv_full + 8 * (14 + b); };
    const uint32_t all_done = kv_full + 8 * 16;
    const uint32_t drain = kv_full + 8 * 17;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kQStages; ++s) {
            mbar_init(q_full0 + 8 * s, 1);
            mbar_init(q_empty0 + 8 * s, 1);
        }
        mbar_init(kv_full, 1);
        for (int h = 0; h < 2; ++h) {
            mbar_init(s_full(h), 1);
            mbar_init(dp_full(h), 1);
            mbar_init(p_full(h), 4);
            mbar_init(ds_full(h), 4);
            mbar_init(s_free(h), 4);
            mbar_init(dv_done(h), 1);
        }
        mbar_init(dq_full, 1);
        mbar_init(dq_free(0), 4);
        mbar_init(dq_free(1), 4);
        mbar_init(all_done, 1);
        mbar_init(drain, 1);
        *abort_flag = 0u;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmKD);
        tma_prefetch_desc(&tmV);
        tma_prefetch_desc(&tmDO);
        tma_prefetch_desc(&tmL);
        tma_prefetch_desc(&tmQaug);
    }
    // Constant value-side slice of the dP MMA: every row [0, 0, 1, 1, 0 ...] (K-major,
    // 32-byte rows, 32-byte swizzle: the two 16-byte chunks of row r swap when bit 2 of r
    // is set).  Against the query slice [1, 1, -delta_hi, -delta_lo, ...] it adds -delta.
    if (threadIdx.x < 2 * kTile) {
        const int r = threadIdx.x >> 1, c = threadIdx.x & 1;
        const int phys = c ^ ((r >> 2) & 1);
        const uint32_t one2 = 0x3C003C00u;  // two fp16 ones
        *reinterpret_cast<uint4*>(smem + Cfg::OFF_VAUG + r * 32 + phys * 16) =
            c == 0 ? make_uint4(0u, one2, 0u, 0u) : make_uint4(0u, 0u, 0u, 0u);
        fence_proxy_async_smem();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), Cfg::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int wgroup = warp >> 2;

    // Each role's code sits inside the branch that adjusts its warpgroup's registers, so
    // the register allocator budgets it with the post-setmaxnreg count.
    if (wgroup == 0) {
      regs_dec<kRegsProducer>();
      if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            const uint32_t sK = smem_u32(smem + Cfg::OFF_K);
            const uint32_t sV = smem_u32(smem + Cfg::OFF_V);
            mbar_arrive_expect_tx(kv_full, 3 * Cfg::KC_BYTES + Cfg::V_BYTES);
            tma_load_3d(sK, &tmK, kv_full, 0, kv0, bh);
            if (Cfg::DQ_MERGED) {
                tma_load_3d(smem_u32(smem + Cfg::OFF_KD), &tmKD, kv_full, 0, kv0, bh);
            } else {  // two 64-column chunks: hi, lo
                tma_load_3d(smem_u32(smem + Cfg::OFF_KD), &tmKD, kv_full, 0, kv0, bh);
                tma_load_3d(smem_u32(smem + Cfg::OFF_KD + Cfg::KC_STRIDE), &tmKD, kv_full, MC, kv0, bh);
            }
            tma_load_3d(sV, &tmV, kv_full, 0, kv0, bh);
            if (HD > 64) tma_load_3d(sV + kTile * 128, &tmV, kv_full, 64, kv0, bh);
            int issued = 0;
            for (int it = 0; it < n_it; ++it) {
                const int s = it % kQStages;
                if (it >= kQStages &&
                    !mbar_wait(q_empty0 + 8 * s, ((it / kQStages) & 1) ^ 1, args.status, K_ATTN_BWD, 1)) {
                    *abort_flag = 1u;
                    break;
                }
                if (*abort_flag) break;
                const int q0 = (i_begin + it) * kTile;
                const uint32_t fb = q_full0 + 8 * s;
                const uint32_t sQ = smem_u32(smem + Cfg::OFF_Q + s * Cfg::KC_STRIDE);
                const uint32_t sDO = smem_u32(smem + Cfg::OFF_DO + s * Cfg::V_BYTES);
                mbar_arrive_expect_tx(fb, Cfg::STAGE_TX);
                tma_load_3d(sQ, &tmQ, fb, 0, q0, bh);
                tma_load_3d(sDO, &tmDO, fb, h * HD, q0, b);
                if (HD > 64) tma_load_3d(sDO + kTile * 128, &tmDO, fb, h * HD + 64, q0, b);
                tma_load_2d(smem_u32(smem + Cfg::OFF_L + s * kTile * 4), &tmL, fb, q0, bh);
                tma_load_3d(smem_u32(smem + Cfg::OFF_QAUG + s * Cfg::AUG_BYTES), &tmQaug, fb, 0, q0, bh);
                ++issued;
            }
            mbar_wait(kv_full, 0, args.status, K_ATTN_BWD, 2);
            if (*abort_flag) {
                for (int i = max(0, issued - kQStages); i < issued; ++i)
                    mbar_wait(q_full0 + 8 * (i % kQStages), (i / kQStages) & 1, args.status, K_ATTN_BWD, 2);
            }
        }
      } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        // The whole warp runs this loop (warp-uniform control flow and descriptor arithmetic);
        // elect.sync inside umma_*_w / umma_commit_w lets one lane issue each instruction.
        {
            constexpr uint32_t id_dv = make_idesc_f16(128, HD, false, true);    // dV
            constexpr uint32_t id_mc = make_idesc_f16(128, MC, false, true);    // dK (A in TMEM)
            constexpr uint32_t id_dq = make_idesc_f16(128, Cfg::DQ_COLS, true, true);  // dQ (A MN-major smem)
            constexpr uint32_t kd_sw = swizzle_code_for_row_bytes(Cfg::KD_ROW);
            constexpr uint32_t kc_sw = swizzle_code_for_row_bytes(Cfg::KC_ROW);
            constexpr uint32_t v_sw = swizzle_code_for_row_bytes(Cfg::V_ROW);
            const uint32_t sK = smem_u32(smem + Cfg::OFF_K);
            const uint32_t sKD = smem_u32(smem + Cfg::OFF_KD);
            const uint32_t sV = smem_u32(smem + Cfg::OFF_V);
            const uint32_t sDS = smem_u32(smem + Cfg::OFF_DS);
            auto qbuf = [&](int it) { return smem_u32(smem + Cfg::OFF_Q + (it % kQStages) * Cfg::KC_STRIDE); };
            auto dobuf = [&](int it) { return smem_u32(smem + Cfg::OFF_DO + (it % kQStages) * Cfg::V_BYTES); };
            auto augbuf = [&](int it) { return smem_u32(smem + Cfg::OFF_QAUG + (it % kQStages) * Cfg::AUG_BYTES); };
            const uint32_t sVaug = smem_u32(smem + Cfg::OFF_VAUG);
            constexpr uint32_t id_h = make_idesc_f16(128, 64, false, false);  // S_h^T, dP_h^T (64 queries)
            // S_h^T = Kc . Qc_h^T = k.q - cb/2 (centered query codes), into TM_S + 64h
            auto issue_s = [&](int it, int h) {
                const uint32_t sQ = qbuf(it) + 64 * h * Cfg::KC_ROW;
#pragma unroll
                for (int ks = 0; ks < MC / 16; ++ks)
                    umma_ss_w(tmem + Cfg::TM_S + 64 * h, kmajor_desc<Cfg::KC_ROW>(sK, ks),
                              kmajor_desc<Cfg::KC_ROW>(sQ, ks), id_h, ks > 0 ? 1u : 0u);
                umma_commit_w(s_full(h));
            };
            // dP_h^T - delta = V . dO_h^T + [0,0,1,1,..] . [1,1,-delta_hi,-delta_lo,..]^T, into TM_DP + 64h
            auto issue_dp = [&](int it, int h) {
                const uint32_t sDO = dobuf(it) + 64 * h * Cfg::V_ROW;
#pragma unroll
                for (int ks = 0; ks < HD / 16; ++ks)
                    umma_ss_w(tmem + Cfg::TM_DP + 64 * h, kmajor_desc<Cfg::V_ROW>(sV, ks),
                              kmajor_desc<Cfg::V_ROW>(sDO, ks), id_h, ks > 0 ? 1u : 0u);
                umma_ss_w(tmem + Cfg::TM_DP + 64 * h, kmajor_desc<32>(sVaug, 0),
                          kmajor_desc<32>(augbuf(it) + 64 * h * 32, 0), id_h, 1u);
                umma_commit_w(dp_full(h));
            };
            // Lockstep mode: S and dP of both halves as one N = 128 product each, every per-half
            // barrier of the pair committed
            constexpr uint32_t id_full = make_idesc_f16(128, 128, false, false);
            auto issue_s_all = [&](int it) {
                const uint32_t sQ = qbuf(it);
#pragma unroll
                for (int ks = 0; ks < MC / 16; ++ks)
                    umma_ss_w(tmem + Cfg::TM_S, kmajor_desc<Cfg::KC_ROW>(sK, ks), kmajor_desc<Cfg::KC_ROW>(sQ, ks),
                              id_full, ks > 0 ? 1u : 0u);
                umma_commit_w(s_full(0));
                umma_commit_w(s_full(1));
            };
            auto issue_dp_all = [&](int it) {
                const uint32_t sDO = dobuf(it);
#pragma unroll
                for (int ks = 0; ks < HD / 16; ++ks)
                    umma_ss_w(tmem + Cfg::TM_DP, kmajor_desc<Cfg::V_ROW>(sV, ks), kmajor_desc<Cfg::V_ROW>(sDO, ks),
                              id_full, ks > 0 ? 1u : 0u);
                umma_ss_w(tmem + Cfg::TM_DP, kmajor_desc<32>(sVaug, 0), kmajor_desc<32>(augbuf(it), 0), id_full, 1u);
                umma_commit_w(dp_full(0));
                umma_commit_w(dp_full(1));
            };
            // dV += P_h^T . dO_h   (P^T of query half h in columns p_col(h) .. +32)
            auto issue_dv = [&](int it, int h) {
                const uint32_t sDO = dobuf(it);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int ks = 4 * h + k;
                    const uint64_t bd = make_sdesc(sDO + ks * 16 * Cfg::V_ROW, kTile * 128, 8 * Cfg::V_ROW, v_sw);
                    umma_ts_w(tmem + Cfg::TM_DV, tmem + Cfg::p_col(h) + k * 8, bd, id_dv,
                              (it > 0 || ks > 0) ? 1u : 0u);
                }
                umma_commit_w(dv_done(h));
            };
            // dK += dS_h^T . Qc_h   (dS_h^T in the first 32 dP_h columns)
            //   (centered codes: this is dk + gate_q * dcb, whose cancelling bias term is exact)
            auto issue_dk = [&](int it, int h) {
                const uint32_t sQ = qbuf(it);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int ks = 4 * h + k;
                    const uint64_t bd = make_sdesc(sQ + ks * 16 * Cfg::KC_ROW, 16, 8 * Cfg::KC_ROW, kc_sw);
                    umma_ts_w(tmem + Cfg::TM_DK, tmem + Cfg::TM_DP + 64 * h + k * 8, bd, id_mc,
                              (it > 0 || ks > 0) ? 1u : 0u);
                }
            };
            // dQ = dS . (k - gate_k/2) with the fp16 hi + lo parts (A = both halves of the shared dS
            // tile, MN-major): one N = 2m MMA whose column halves the dQ warps add, or two
            // accumulating N = m passes; then the tile's stage is free
            auto issue_dq = [&](int it) {
                const uint32_t sDSi = sDS + (it % Cfg::N_DS) * Cfg::DS_BYTES;
#pragma unroll
                for (int part = 0; part < (Cfg::DQ_MERGED ? 1 : 2); ++part) {
                    const uint32_t sKd = sKD + part * Cfg::KC_STRIDE;
#pragma unroll
                    for (int ks = 0; ks < kTile / 16; ++ks) {
                        const uint64_t ad = make_sdesc(sDSi + ks * 2048, kTile * 128, 1024, SW_128);
                        const uint64_t bd = make_sdesc(sKd + ks * 16 * Cfg::KD_ROW, 16, 8 * Cfg::KD_ROW, kd_sw);
                        umma_ss_w(tmem + Cfg::TM_DQ, ad, bd, id_dq, (part > 0 || ks > 0) ? 1u : 0u);
                    }
                }
                umma_commit_w(dq_full);  // also: the shared dS tile is free again
                umma_commit_w(q_empty0 + 8 * (it % kQStages));
            };
            auto wait = [&](uint32_t bar, int phase, uint32_t site) {
                if (!mbar_wait_warp(bar, static_cast<uint32_t>(phase) & 1u, args.status, K_ATTN_BWD, site))
                    return false;
                tc_fence_after();
                return true;
            };
            // Issue order per iteration i (half 1 runs half a tile behind half 0; tcgen05.mma from
            // one thread execute in order):
            //   A  dV_1(i-1)                      [then S_1(i) when P shares S's columns]
            //   B  S_0(i+1) once half 0 holds S_0(i)          (P in its own columns)
            //   C  dK_1(i-1), dQ(i-1), dP_1(i)   (dP_1 overwrites dS_1 after dK_1 read it)
            //   D  dV_0(i)                        [then S_0(i+1) when P shares S's columns]
            //   E  S_1(i+1) once half 1 holds S_1(i)           (P in its own columns)
            //   F  dK_0(i), dP_0(i+1)
            // S_h(i+1) is issued only once stage i+1 has landed (waited for here; the softmax warps'
            // arrivals do not imply it), and every later use of that stage follows in issue order.
            // With fewer than 3 stages, stage i+1 is the one C releases (tile i-1), so C goes first.
            constexpr bool kCFirst = kQStages < 3;
            auto stage_landed = [&](int it2) { return wait(q_full0 + 8 * (it2 % kQStages), it2 / kQStages, 17); };
            bool ok = wait(kv_full, 0, 3);
            if (ok && n_it > 0) {
                ok = wait(q_full0, 0, 4);
                if (ok && SPLIT) {
                    issue_s(0, 0);
                    issue_s(0, 1);
                    issue_dp(0, 0);
                    issue_dp(0, 1);
                } else if (ok) {
                    issue_s_all(0);
                    issue_dp_all(0);
                }
            }
            // Lockstep mode (few query tiles per CTA, or one dS tile, where the halves would not
            // stay apart): per tile i, S_{i+1} once both halves hold S_i, dV_i once both P halves
            // are in TMEM, then dK_i, dQ_i and dP_{i+1} once both dS halves are written.
            for (int it = 0; !SPLIT && ok && it < n_it; ++it) {
                const bool nxt = it + 1 < n_it;
                if (Cfg::P_SEP && nxt) {
                    if (!(ok = wait(s_free(0), it, 15) && wait(s_free(1), it, 15) && stage_landed(it + 1))) break;
                    issue_s_all(it + 1);
                }
                if (!(ok = wait(p_full(0), it, 5) && wait(p_full(1), it, 5))) break;
                issue_dv(it, 0);
                issue_dv(it, 1);
                if (!Cfg::P_SEP && nxt) {
                    if (!(ok = stage_landed(it + 1))) break;
                    issue_s_all(it + 1);
                }
                if (!(ok = wait(ds_full(0), it, 6) && wait(ds_full(1), it, 6))) break;
                issue_dk(it, 0);
                issue_dk(it, 1);
                if (Cfg::DS2 && it >= 1 && !(ok = wait(dq_free((it - 1) % 2), (it - 1) / 2, 19))) break;
                issue_dq(it);
                if (nxt) issue_dp_all(it + 1);
            }
            for (int it = 0; SPLIT && ok && it <= n_it; ++it) {
                const bool cur = it < n_it, nxt = it + 1 < n_it, prev = it > 0;
                if (prev) {  // A
                    if (!(ok = wait(p_full(1), it - 1, 5))) break;
                    issue_dv(it - 1, 1);
                    if (!Cfg::P_SEP && cur) issue_s(it, 1);
                }
                auto step_c = [&]() {
                    if (!wait(ds_full(1), it - 1, 6)) return false;
                    issue_dk(it - 1, 1);
                    // with two dS tiles the softmax warps no longer wait for dQ_{i-2} to be read out
                    // of TMEM before writing dS_{i-1}: the dQ accumulator's release is waited for here
                    if (Cfg::DS2 && it >= 2 && !wait(dq_free((it - 2) % 2), (it - 2) / 2, 19)) return false;
                    issue_dq(it - 1);
                    if (cur) issue_dp(it, 1);
                    return true;
                };
                if (kCFirst && prev && !(ok = step_c())) break;
                if (Cfg::P_SEP && nxt) {  // B
                    if (!(ok = wait(s_free(0), it, 15) && stage_landed(it + 1))) break;
                    issue_s(it + 1, 0);
                }
                if (!kCFirst && prev && !(ok = step_c())) break;  // C
                if (!cur) break;
                if (!(ok = wait(p_full(0), it, 5))) break;  // D
                issue_dv(it, 0);
                if (!Cfg::P_SEP && nxt) {
                    if (!(ok = stage_landed(it + 1))) break;
                    issue_s(it + 1, 0);
                }
                if (Cfg::P_SEP && nxt) {  // E
                    if (!(ok = wait(s_free(1), it, 15))) break;
                    issue_s(it + 1, 1);
                }
                if (!(ok = wait(ds_full(0), it, 6))) break;  // F
                issue_dk(it, 0);
                if (nxt) issue_dp(it + 1, 0);
            }
            if (ok) {
                umma_commit_w(all_done);
            } else {
                *abort_flag = 1u;
                umma_commit_w(drain);
                mbar_wait_warp(drain, 0, args.status, K_ATTN_BWD, 8);
                umma_commit_w(all_done);  // release the epilogue waits
            }
        }
      }
    } else if (wgroup == 1 || wgroup == 2) {
        regs_inc<kRegsSoftmax>();
        // ---------------- softmax warps (4..11) ----------------
        const int wg = wgroup - 1;        // 0: queries [0,64), 1: queries [64,128)
        const int quad = warp & 3;
        const int j = quad * 32 + lane;   // key row within the tile
        const int kv = kv0 + j;
        const bool kv_ok = kv < args.N;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
        const float c2 = args.c2;
        uint8_t* ds_row = smem + Cfg::OFF_DS + wg * (kTile * 128) + j * 128;
        const int sw = j & 7;
        float dcb = 0.f;
        bool ok = true;
        // half 1 starts half a tile behind half 0 (once half 0 has its first P), so that the two
        // warpgroups' exponential and dS phases alternate on every sub-partition
        if (SPLIT && wg == 1 && n_it > 1 && !mbar_wait_warp(p_full(0), 0, args.status, K_ATTN_BWD, 18)) ok = false;
        for (int it = 0; ok && it < n_it; ++it) {
            const int s = it % kQStages;
            const int q0 = (i_begin + it) * kTile;
            const int qc0 = q0 + wg * 64;  // first query of this warp group's half
            // S_h(i) ready; stage i landed (the MMA thread waited for it before issuing S_h(i), so
            // this returns at once; it orders this warp's reads of L_i after the TMA's write)
            if (!mbar_wait_warp(s_full(wg), it & 1, args.status, K_ATTN_BWD, 9) ||
                !mbar_wait_warp(q_full0 + 8 * s, (it / kQStages) & 1, args.status, K_ATTN_BWD, 10)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const float4* Lv = reinterpret_cast<const float4*>(smem + Cfg::OFF_L + s * kTile * 4) + wg * 16;
            const bool need_mask =
                !kv_ok || (qc0 + 64 > args.N) || (CAUSAL && qc0 < kv0 + kTile) || (args.mask_diag && q0 == kv0);
            // P^T = 2^(c2 * (k.q - cb/2) - L_i): both TMEM loads in flight before one wait
            float p[64];
            {
                uint32_t rr[64];
                tmem_ld32(lane_base + Cfg::TM_S + wg * 64, rr);
                tmem_ld32(lane_base + Cfg::TM_S + wg * 64 + 32, rr + 32);
                tmem_ld_wait();
                // s_free_h(i): S_h(i+1) may overwrite these columns
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(s_free(wg));
#pragma unroll
                for (int i = 0; i < 64; i += 4) {
                    const float4 L = Lv[i / 4];
                    p[i] = ex2(fmaf(u2f(rr[i]), c2, -L.x));
                    p[i + 1] = ex2(fmaf(u2f(rr[i + 1]), c2, -L.y));
                    p[i + 2] = ex2(fmaf(u2f(rr[i + 2]), c2, -L.z));
                    p[i + 3] = ex2(fmaf(u2f(rr[i + 3]), c2, -L.w));
                }
            }
            if (need_mask) {
#pragma unroll
                for (int c = 0; c < 64; ++c) {
                    const int qi = qc0 + c;
                    const bool keep = kv_ok && qi < args.N && (!CAUSAL || kv <= qi) && !(args.mask_diag && kv == qi);
                    p[c] = keep ? p[c] : 0.f;
                }
            }
            if (Cfg::P_SEP && it > 0) {  // the P columns hold P_{i-1} until dV_{i-1} has read it
                if (!mbar_wait_warp(dv_done(wg), (it - 1) & 1, args.status, K_ATTN_BWD, 16)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
            }
            {
                uint32_t pk[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) pk[i] = pack_half2(p[2 * i], p[2 * i + 1]);
                tmem_st16(lane_base + Cfg::p_col(wg), pk);
                tmem_st16(lane_base + Cfg::p_col(wg) + 16, pk + 16);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full(wg));

            if (!mbar_wait_warp(dp_full(wg), it & 1, args.status, K_ATTN_BWD, 11)) {
                ok = false;
                break;
            }
            tc_fence_after();
            // dS^T = P^T (dP^T - delta); the MMA already subtracted delta
            {
                uint32_t rr[64];
                tmem_ld32(lane_base + Cfg::TM_DP + wg * 64, rr);
                tmem_ld32(lane_base + Cfg::TM_DP + wg * 64 + 32, rr + 32);
                tmem_ld_wait();
                uint32_t pk[32];
#pragma unroll
                for (int i = 0; i < 64; i += 2) {
                    const float d0 = p[i] * u2f(rr[i]);
                    const float d1 = p[i + 1] * u2f(rr[i + 1]);
                    dcb += d0 + d1;
                    pk[i / 2] = pack_half2(d0, d1);
                }
                tmem_st16(lane_base + Cfg::TM_DP + wg * 64, pk);
                tmem_st16(lane_base + Cfg::TM_DP + wg * 64 + 16, pk + 16);
                // smem copy for the dQ MMA into dS tile b = i % N_DS: row j, 16-byte units u = 0..7,
                // 128-byte swizzle, once the tile's previous user (query tile i - N_DS) is done:
                // dq_free(b) comes after the dQ MMA read it, the dQ warps read that dQ out of TMEM
                // and the TMA read what they staged there.  (With one tile that is dQ_{i-1}, and
                // ds_full(i) then also tells the MMA thread that the dQ accumulator is free.)
                const int b = it % Cfg::N_DS;
                if (it >= Cfg::N_DS &&
                    !mbar_wait_warp(dq_free(b), (it / Cfg::N_DS - 1) & 1, args.status, K_ATTN_BWD, 7)) {
                    ok = false;
                    break;
                }
                uint8_t* ds_dst = ds_row + b * Cfg::DS_BYTES;
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    *reinterpret_cast<uint4*>(ds_dst + ((u ^ sw) << 4)) =
                        make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
            }
            tmem_st_wait();
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(ds_full(wg));
        }
        // ---- epilogue: dV (group 0), dK + dcb (group 1)
        float* dcb_x = reinterpret_cast<float*>(smem + Cfg::OFF_DCB);
        if (wg == 1) dcb_x[j] = dcb;
        asm volatile("bar.sync 1, 256;" ::: "memory");
        const bool fin = ok && mbar_wait_warp(all_done, 0, args.status, K_ATTN_BWD, 13) && !*abort_flag;
        if (fin) {
            tc_fence_after();
            const size_t tok = static_cast<size_t>(b) * args.N + kv;
            if (wg == 0) {
                __half* dst = args.dcat + tok * args.Cp + args.Hp + h * HD;
#pragma unroll
                for (int c = 0; c < HD; c += 16) {
                    uint32_t rr[16];
                    tmem_ld16(lane_base + Cfg::TM_DV + c, rr);
                    tmem_ld_wait();
                    if (kv_ok) {
                        uint4* d4 = reinterpret_cast<uint4*>(dst + c);
                        d4[0] = make_uint4(pack_half2(u2f(rr[0]), u2f(rr[1])), pack_half2(u2f(rr[2]), u2f(rr[3])),
                                           pack_half2(u2f(rr[4]), u2f(rr[5])), pack_half2(u2f(rr[6]), u2f(rr[7])));
                        d4[1] = make_uint4(pack_half2(u2f(rr[8]), u2f(rr[9])), pack_half2(u2f(rr[10]), u2f(rr[11])),
                                           pack_half2(u2f(rr[12]), u2f(rr[13])),
                                           pack_half2(u2f(rr[14]), u2f(rr[15])));
                    }
                }
                if (kv_ok) args.dcb[static_cast<size_t>(bh) * args.Npad + kv] = args.neg_scale * (dcb + dcb_x[j]);
            } else {
                float* dst = args.dk + (static_cast<size_t>(bh) * args.N + kv) * MC;
#pragma unroll
                for (int c = 0; c < MC; c += 16) {
                    uint32_t rr[16];
                    tmem_ld16(lane_base + Cfg::TM_DK + c, rr);
                    tmem_ld_wait();
                    if (kv_ok) {
                        float4* d4 = reinterpret_cast<float4*>(dst + c);
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            d4[i] = make_float4(u2f(rr[4 * i]) * args.two_scale, u2f(rr[4 * i + 1]) * args.two_scale,
                                                u2f(rr[4 * i + 2]) * args.two_scale,
                                                u2f(rr[4 * i + 3]) * args.two_scale);
                    }
                }
            }
        } else {
            *abort_flag = 1u;
        }
    } else {
        regs_dec<kRegsDq>();
        // ---------------- dQ warps (12..15) ----------------
        const int quad = warp & 3;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
        // Staging: this warp's 32 rows in the shared dS tile, as DQ_BOXES boxes of 32 rows x
        // DQ_BOX fp32 columns in the TMA swizzle of the dq tensor map (128 B rows: 16-byte unit
        // u of row r at u ^ (r & 7); 64 B rows: u ^ ((r >> 1) & 3)).  The tile is free from
        // dq_full(i) (the dQ MMA has read dS_i) until dq_free(i), which this warpgroup gives
        // only once the TMA has read the staged rows.
        constexpr int DQ_BOX = MC < 32 ? MC : 32;
        constexpr int DQ_BOXES = MC / DQ_BOX;
        constexpr int DQ_ROWB = DQ_BOX * 4;
        static_assert(4 * DQ_BOXES * 32 * DQ_ROWB <= Cfg::DS_BYTES, "dQ staging fits the dS tile");
        const uint32_t stage0 = smem_u32(smem + Cfg::OFF_DS + quad * (DQ_BOXES * 32 * DQ_ROWB));
        const int swz = DQ_ROWB == 128 ? (lane & 7) : ((lane >> 1) & 3);
        for (int it = 0; it < n_it; ++it) {
            if (!mbar_wait_warp(dq_full, it & 1, args.status, K_ATTN_BWD, 14) || *abort_flag) break;
            tc_fence_after();
            const int q0 = (i_begin + it) * kTile + quad * 32;  // first row of this warp
            const uint32_t stage = stage0 + (it % Cfg::N_DS) * Cfg::DS_BYTES;  // the dS tile dQ_i read
            const uint32_t my_row = stage + lane * DQ_ROWB;
#pragma unroll 1
            for (int c = 0; c < MC; c += 16) {
                uint32_t rr[16];
                tmem_ld16(lane_base + Cfg::TM_DQ + c, rr);
                if (Cfg::DQ_MERGED) {  // add the lo half
                    uint32_t lo[16];
                    tmem_ld16(lane_base + Cfg::TM_DQ + MC + c, lo);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 16; ++i) rr[i] = __float_as_uint(u2f(rr[i]) + u2f(lo[i]));
                } else {
                    tmem_ld_wait();
                }
                const uint32_t row = my_row + (c / DQ_BOX) * (32 * DQ_ROWB);
                const int u0 = (c % DQ_BOX) / 4;
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    st_shared_v4(row + (((u0 + k) ^ swz) << 4), u2f(rr[4 * k]) * args.two_scale,
                                 u2f(rr[4 * k + 1]) * args.two_scale, u2f(rr[4 * k + 2]) * args.two_scale,
                                 u2f(rr[4 * k + 3]) * args.two_scale);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0 && q0 < args.N) {  // rows past N are clipped by the TMA
#pragma unroll
                for (int bx = 0; bx < DQ_BOXES; ++bx)
                    tma_reduce_add_3d(&tmDQ, stage + bx * (32 * DQ_ROWB), bx * DQ_BOX, q0, bh);
                bulk_commit_group();
                bulk_wait_read_all();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(dq_free(it % Cfg::N_DS));
        }
        if (lane == 0) bulk_wait_all();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::TMEM_COLS);
    }
}

template <int MC, int HD, bool CAUSAL>
int run_bwd(const DeviceInfo& dev, const Shape& s, const ProjOut& p, const AttnBwdIO& io, cudaStream_t stream) {
    using Cfg = BwdCfg<MC, HD>;
    const int BH = s.B * s.H;
    const int Npad = (s.N + kTile - 1) / kTile * kTile;
    CUtensorMap tQ, tK, tKD, tV, tDO, tL, tQA, tDQ;
    if (p.kdq == nullptr || io.qaug == nullptr)
        return set_error(MORPHO_ERR_INVALID, "internal: backward needs the centered key codes and bias slices");
    MORPHO_TRY(make_tmap_3d_f16(&tQ, p.qc, MC, s.N, BH, MC, static_cast<uint64_t>(s.N) * MC, MC, kTile));
    MORPHO_TRY(make_tmap_3d_f16(&tK, p.kc, MC, s.N, BH, MC, static_cast<uint64_t>(s.N) * MC, MC, kTile));
    MORPHO_TRY(make_tmap_3d_f16(&tKD, p.kdq, 2 * MC, s.N, BH, 2 * MC, static_cast<uint64_t>(s.N) * 2 * MC,
                                Cfg::DQ_MERGED ? 2 * MC : MC, kTile));
    MORPHO_TRY(make_tmap_3d_f16(&tV, p.v, HD, s.N, BH, HD, static_cast<uint64_t>(s.N) * HD, HD > 64 ? 64 : HD,
                                kTile));
    MORPHO_TRY(make_tmap_3d_f16(&tDO, io.dO, s.D, s.N, s.B, s.D, static_cast<uint64_t>(s.N) * s.D,
                                HD > 64 ? 64 : HD, kTile));
    MORPHO_TRY(make_tmap_2d_f32(&tL, io.L, BH, Npad, Npad, 1, kTile));
    MORPHO_TRY(make_tmap_3d_f16(&tQA, io.qaug, 16, s.N, BH, 16, static_cast<uint64_t>(s.N) * 16, 16, kTile));
    {  // dq [BH, N, MC] fp32, reduced into by 32-row boxes of up to 32 columns
        const uint64_t dims[3] = {static_cast<uint64_t>(MC), static_cast<uint64_t>(s.N), static_cast<uint64_t>(BH)};
        const uint64_t strides[2] = {static_cast<uint64_t>(MC) * 4, static_cast<uint64_t>(s.N) * MC * 4};
        const uint32_t box[3] = {MC < 32 ? MC : 32u, 32u, 1u};
        MORPHO_TRY(make_tmap(&tDQ, io.dq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, dims, strides, box,
                             MC < 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B));
    }
    BwdArgs a;
    a.N = s.N;
    a.Npad = Npad;
    a.H = s.H;
    a.D = s.D;
    a.Hp = s.Hp();
    a.Cp = s.Cp();
    a.n_qtiles = Npad / kTile;
    a.mask_diag = s.mask_diag ? 1 : 0;
    a.c2 = 2.0f * s.scale * kLog2e;
    a.two_scale = 2.0f * s.scale;
    a.neg_scale = -s.scale;
    a.cb = p.cb;
    a.dcat = io.dcat;
    a.dk = io.dk;
    a.dcb = io.dcb;
    a.dq = io.dq;
    a.status = dev.status;
    // The half-tile pipelines pay for their split MMAs only where the halves stay apart: with two
    // dS tiles and enough query tiles per CTA to amortise the offset start; else lockstep.
    constexpr int kSplitMinTiles = 16;
    const bool split = Cfg::DS2 && a.n_qtiles >= kSplitMinTiles;
    auto kern = split ? attn_bwd_kernel<MC, HD, CAUSAL, true> : attn_bwd_kernel<MC, HD, CAUSAL, false>;
    MORPHO_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES));
    a.BH = BH;
    a.band = causal_band(static_cast<long long>(s.N) * (2 * MC + 2 * HD + 36), BH, a.n_qtiles);
    const dim3 grid = CAUSAL ? dim3(a.n_qtiles * BH, 1) : dim3(a.n_qtiles, BH);
    prof_begin(stream, "attn_bwd");
    kern<<<grid, kBwdThreads, Cfg::SMEM_BYTES, stream>>>(tQ, tK, tKD, tV, tDO, tL, tQA, tDQ, a);
    MORPHO_LAUNCH_CHECK("attn_bwd");
    return MORPHO_OK;
}

template <int MC, int HD>
int run_bwd_c(const DeviceInfo& dev, const Shape& s, const ProjOut& p, const AttnBwdIO& io, cudaStream_t st) {
    return s.causal ? run_bwd<MC, HD, true>(dev, s, p, io, st) : run_bwd<MC, HD, false>(dev, s, p, io, st);
}

template <int MC>
int run_bwd_hd(const DeviceInfo& dev, const Shape& s, const ProjOut& p, const AttnBwdIO& io, cudaStream_t st) {
    switch (s.hd) {
        case 32: return run_bwd_c<MC, 32>(dev, s, p, io, st);
        case 64: return run_bwd_c<MC, 64>(dev, s, p, io, st);
        case 128: return run_bwd_c<MC, 128>(dev, s, p, io, st);
        default: return set_error(MORPHO_ERR_INVALID, "head_dim %d not supported (32, 64 or 128)", s.hd);
    }
}

}  // namespace

int launch_attn_bwd(const DeviceInfo& dev, const Shape& s, const ProjOut& p, const AttnBwdIO& io,
                    cudaStream_t stream) {
    switch (s.m) {
        case 16: return run_bwd_hd<16>(dev, s, p, io, stream);
        case 32: return run_bwd_hd<32>(dev, s, p, io, stream);
        case 64: return run_bwd_hd<64>(dev, s, p, io, stream);
        default: return set_error(MORPHO_ERR_INVALID, "cube_m %d not supported (16, 32 or 64)", s.m);
    }
}

}  // namespace morpho

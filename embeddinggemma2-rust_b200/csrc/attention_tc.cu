// Varlen packed flash attention on tcgen05 for the text backbone: bidirectional, scale 1,
// inclusive sliding window (radius `window`) or global, block-diagonal over packed sequences.
//
// Replaces the reference's bf16 flash kernels `flash_attn_d256_packed_bb` and `flash_attn_d512_bb`
// (kernels_sm80.cu:236-416, :474-684; mma.sync) and their launchers (src/gpu/mod.rs:1217-1241,
// :1547-1599); semantics of src/ops.rs:364-444.
//
// Query tiles pack the G = nh / nkv query heads that share a K/V head into the 128 MMA rows of a
// CTA: row r = token (r / G), head (g * G + r % G), so each K/V tile loaded serves all G heads
// (sliding layers, G = 2: 64 tokens per CTA; global layers, G = 4: 32). Softmax: one thread per
// row, online max / sum in the log2 domain with the log2(e) scale folded into one FFMA, O rescaled in
// TMEM only when a row max grows by more than 2^8 (else the stale max is kept, which is exact), P
// written to TMEM as packed bf16 and read from there by the P V MMA; at the end O / l is stored as
// bf16.
#include "common.cuh"
#include "kernels.h"

namespace eg2 {

constexpr int ATT_KBOX = 64;   // keys per K box (one CTA's half of a 128-key tile)
constexpr int ATT_DV = 256;    // output channels per cluster
constexpr float ATT_RESCALE_LOG2 = 8.f;

struct AttParams {
    const AttnTile* tiles;
    bf16_t* out;
    const int* seq_start;  // per row: first row of its sequence (null: a tile's rows are one sequence)
    const int* seq_len;
    const bf16_t* q;  // [rows, nh, hd] (read directly by the head-512 kernel, which keeps Q in TMEM)
    long rows;
    int nh, nkv, hd, window, G, tq, nsplit, n_tiles;
};

// ---------------------------------------------------------------------------------------------
// CTA pairs (cta_group::2) over 128-key tiles, head 256 and head 512.
//
// A 2-CTA cluster takes two adjacent query tiles of one sequence and K/V head (128 MMA rows each)
// and runs every MMA as one M = 256 tcgen05.mma issued by the even CTA: S = Q K^T at N = 128 keys
// (each CTA holds 64 of them) and O += P V at N = 256 channels (each CTA holds V for 128 of them).
// Each CTA therefore loads and feeds the tensor cores half of every K / V tile, which halves the
// shared-memory traffic per FLOP of a single-CTA kernel (there: 320 KB per 128-key tile against
// 128 B/cycle of shared memory for 2,048 tensor cycles; here 192 KB). Keys span the union of both
// tiles' windows; each row masks its own. Head 512: O is produced 256 channels at a time, so two
// clusters share each pair of query tiles (one per channel half), each computing the full S.
//
// TMEM per CTA, O at [256, 512). Head 512 (SDB): two S buffers [0, 128) and [128, 256); tile T's S
// goes to buffer T % 2 and its P (packed bf16, 64 columns) over the first half of that S once the
// softmax has read it, so S(T + 1) is computed while the softmax works on T and S(T) waits only for
// P V(T - 2), the last reader of its buffer (the tensor work per tile, 3,072 cycles, exceeds the
// softmax's). Head 256: one S [0, 128) and P[0] [128, 192), P[1] [192, 256); S(T) waits until the
// softmax has read S(T - 1) (s_empty) -- its softmax takes about as long as its 2,048 cycles of
// tensor work, and chaining P V(T - 2) -> S(T) measured 15% slower. Per CTA shared memory: Q (64 / 128 KB) and a ring of 32 KB units (4 / 3), consumed
// in order K(j + 1), V(j); a K unit is 64 keys x 256 channels (head 512: two per tile), a V unit 128
// keys x 128 channels. The even CTA's barriers collect both CTAs' TMA bytes (q_full, r_full) and both
// CTAs' softmax arrivals (p_full, o_empty: 256); MMA completion is committed to the barriers of both
// CTAs (r_empty, s_full, pv_done, q_empty).
//
//   warp 0      TMA producer (this CTA's Q and its half of every unit)
//   warp 1      TMEM allocation (both CTAs); in the even CTA lane 0 issues the S = Q K^T MMAs
//   softmax     head 256: warps 2..9, two threads per row (64 of the 128 columns each; the pair
//               swaps its row maxima through shared memory with a bounded mbarrier handshake, so
//               both take the same stale-max decisions, and adds the row sums at the end); head 512:
//               warps 2..5, one thread per row. O / l epilogue
//   last warp   in the even CTA lane 0 issues the O += P V MMAs
// Two issuing threads: tcgen05.mma issue blocks once a couple of MMAs are queued, so one thread
// leaves the tensor pipe idle during each of its waits and commits; with S and P V on different
// threads (disjoint TMEM, per-thread commit tracking) one feeds the pipe while the other waits.
// ---------------------------------------------------------------------------------------------
constexpr int AP_BN = 128;
constexpr int AP_UNIT = 32768;
template <int DQK>
struct ApCfg {
    static constexpr bool SPLIT = DQK == 256;        // two softmax threads per row
    static constexpr int NSW = SPLIT ? 8 : 4;        // softmax warps
    static constexpr int PV_WARP = 2 + NSW;
    static constexpr int THREADS = 32 * (PV_WARP + 1);
    static constexpr int QCH = DQK / 64;             // Q chunks of [128 rows x 64 channels]
    static constexpr int KU = DQK / 256;             // K units per key tile
    static constexpr int Q_BYTES = QCH * 128 * 128;
    static constexpr int UNITS = DQK == 256 ? 4 : 3;
    static constexpr int OFF_R = Q_BYTES;
    static constexpr int OFF_BAR = OFF_R + UNITS * AP_UNIT;
    // q, ring full/empty, s_full[2], s_empty, p[2], pv[2], drain[2], q_empty, o_empty; split softmax:
    // pair handshakes [4 quadrants][2]
    static constexpr int N_BARS = 1 + 2 * UNITS + 3 + 4 + 2 + 2 + (SPLIT ? 8 : 0);
    static constexpr int OFF_X = OFF_BAR + N_BARS * 8 + 16;  // split softmax: maxima [2 slots][2 halves][128], sums [2][128]
    // Head 256: per softmax warp a 2 KB staging tile for the O epilogue's TMA stores (1 KB aligned).
    static constexpr int OFF_STG = SPLIT ? ((OFF_X + 3 * 1024 + 1023) / 1024) * 1024 : OFF_X;
    static constexpr int SMEM = 1024 + OFF_STG + (SPLIT ? NSW * 2048 : 0);
};
static_assert(ApCfg<256>::SMEM <= 227 * 1024 && ApCfg<512>::SMEM <= 227 * 1024, "attention pair: shared memory");

// Persistent: each cluster walks work units u = cluster, cluster + clusters, ... (a unit is one
// (pair tile, K/V head, 256-channel half of O)), keeping its barriers, K/V ring and TMEM. Across a
// unit boundary the next unit's Q load (once every S MMA of the previous unit has completed:
// q_empty) and its first S = Q K^T run under the previous unit's last P V and O epilogue; its first
// P V waits until the softmax threads have read O out (o_empty). Barrier phases follow running
// counts: T = key tiles so far (s_full, p_full, pv_done), X = split-softmax handshakes,
// U = units with keys so far (q_full, q_empty, o_empty); units without keys are skipped by every role.
template <int DQK>
__global__ void __launch_bounds__(ApCfg<DQK>::THREADS, 1)
    attention_pair_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, AttParams prm) {
    using Cfg = ApCfg<DQK>;
    constexpr bool SPLIT = Cfg::SPLIT;
    constexpr bool SDB = DQK == 512;  // double-buffered S, P over S
    constexpr int SM_ARRIVALS = 2 * 32 * Cfg::NSW;  // softmax threads of both CTAs
    constexpr int AP_UNITS = Cfg::UNITS;
    constexpr int KU = Cfg::KU;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
    uint64_t* q_full = bars;
    uint64_t* r_full = bars + 1;
    uint64_t* r_empty = r_full + AP_UNITS;
    uint64_t* s_full = r_empty + AP_UNITS;  // [2]: S buffer (head 256: [0] only)
    uint64_t* s_empty = s_full + 2;         // head 256: S read by both CTAs' softmax threads
    uint64_t* p_full = s_empty + 1;
    uint64_t* pv_done = p_full + 2;
    uint64_t* drain = pv_done + 2;
    uint64_t* q_empty = drain + 2;
    uint64_t* o_empty = q_empty + 1;
    uint64_t* xpair = o_empty + 1;  // split softmax: [quadrant][slot], 64 arrivals (the row's two warps)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::N_BARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool even = rank == 0;
    const int n_units = prm.n_tiles * prm.nkv * prm.nsplit;
    const int u_first = (int)(blockIdx.x >> 1), u_step = (int)(gridDim.x >> 1);
    const int G = prm.G, W = prm.window, tqc = prm.tq;
    // Unit geometry: K/V head g, O half dsplit, the pair tile, this CTA's first query token, key range.
    struct Unit {
        AttnTile tile;
        int g, dsplit, q0r, k_lo, n_kt;
    };
    auto unit_at = [&](int cid) {
        Unit x;
        const int tile_idx = cid / (prm.nkv * prm.nsplit);
        const int rem = cid % (prm.nkv * prm.nsplit);
        x.g = rem / prm.nsplit;
        x.dsplit = rem % prm.nsplit;
        x.tile = prm.tiles[tile_idx];
        x.q0r = x.tile.q0 + (int)rank * tqc;
        const int q_last = min(x.tile.q0 + 2 * tqc, x.tile.len) - 1;
        x.k_lo = (W >= 0) ? max(0, x.tile.q0 - W) : 0;
        const int k_hi = (W >= 0) ? min(x.tile.len, q_last + W + 1) : x.tile.len;
        x.n_kt = x.tile.len > 0 ? (k_hi - x.k_lo + AP_BN - 1) / AP_BN : 0;
        return x;
    };

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int u = 0; u < AP_UNITS; u++) {
            mbar_init(&r_full[u], 1);
            mbar_init(&r_empty[u], 1);
        }
        mbar_init(&s_full[0], 1);
        mbar_init(&s_full[1], 1);
        mbar_init(s_empty, SM_ARRIVALS);
        for (int b = 0; b < 2; b++) {
            mbar_init(&p_full[b], SM_ARRIVALS);
            mbar_init(&pv_done[b], 1);
        }
        mbar_init(q_empty, 1);
        mbar_init(o_empty, SM_ARRIVALS);
        if constexpr (SPLIT)
            for (int x = 0; x < 8; x++) mbar_init(&xpair[x], 64);
        mbar_init(&drain[0], 1);
        mbar_init(&drain[1], 1);
        *abort_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) tmem_alloc_pair(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // Both CTAs' barriers are initialised (and TMEM allocated) before either CTA touches the other's.
    cluster_sync();
    // Programmatic dependent launch: q / k / v and the tile list are read only after the previous
    // kernel has completed.
    grid_dep_launch();
    grid_dep_wait();
    const uint32_t tmem = *tmem_slot;
    const uint32_t t_s = tmem;  // SDB: S / P buffer b at t_s + 128 b; else S at t_s, P[b] at t_p + 64 b
    const uint32_t t_p = tmem + 128;
    const uint32_t t_o = tmem + 256;
    auto on_even = [&](uint64_t* b) { return mapa_shared(smem_u32(b), 0); };

    if (warp == 0) {
        if (lane == 0) {
            int u = 0;
            uint32_t uph = 0;
            int U = 0;
            for (int cid = u_first; cid < n_units; cid += u_step) {
                const Unit x = unit_at(cid);
                if (x.n_kt == 0) continue;
                // K unit ku of key tile jt: this CTA's 64 keys, channels [256 ku, 256 ku + 256), 4 boxes
                // of [64 keys x 64 channels]. V unit: all 128 keys for this CTA's 128 channels of the O
                // half, 2 boxes of [128 keys x 64 channels].
                auto load_unit = [&](int ku, int jt) -> bool {
                    if (!mbar_wait(&r_empty[u], uph ^ 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) return false;
                    if (even) mbar_arrive_expect_tx(&r_full[u], 2 * AP_UNIT);
                    const uint32_t bar = on_even(&r_full[u]);
                    uint8_t* dst = smem + Cfg::OFF_R + u * AP_UNIT;
                    const int key0 = x.tile.row0 + x.k_lo + jt * AP_BN;
                    if (ku >= 0) {
                        for (int c = 0; c < 4; c++)
                            tma_load_3d_pair(dst + c * 8192, &tmK, bar, ku * 256 + c * 64, x.g, key0 + 64 * (int)rank);
                    } else {
                        for (int c = 0; c < 2; c++)
                            tma_load_3d_pair(dst + c * 16384, &tmV, bar, x.dsplit * ATT_DV + (2 * (int)rank + c) * 64, x.g,
                                             key0);
                    }
                    if (++u == AP_UNITS) {
                        u = 0;
                        uph ^= 1;
                    }
                    return true;
                };
                for (int ku = 0; ku < KU; ku++)
                    if (!load_unit(ku, 0)) goto done;
                // Q: once every S MMA of the previous unit has completed.
                if (U > 0 && !mbar_wait(q_empty, (U - 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                if (even) mbar_arrive_expect_tx(q_full, 2 * Cfg::Q_BYTES);
                const uint32_t qbar = on_even(q_full);
                for (int c = 0; c < Cfg::QCH; c++)
                    tma_load_3d_pair(smem + c * 128 * 128, &tmQ, qbar, c * 64, x.g * G, x.tile.row0 + x.q0r);
                for (int j = 0; j < x.n_kt; j++) {
                    if (j + 1 < x.n_kt)
                        for (int ku = 0; ku < KU; ku++)
                            if (!load_unit(ku, j + 1)) goto done;
                    if (!load_unit(-1, j)) goto done;
                }
                U++;
            }
        }
    } else if (warp == 1 || warp == Cfg::PV_WARP) {
        if (even && lane == 0) {
            // Ring position (within a unit, from its first unit) of K(j) unit ku / V(j): the producer's
            // order is K(0), then per tile j K(j + 1) (if any) and V(j); a unit takes n_kt (KU + 1).
            int base = 0, T = 0, U = 0;
            if (warp == 1) {
                constexpr uint32_t idesc_s = umma_idesc(256, AP_BN, 1);
                const uint64_t dq0 = umma_desc_sw128(smem_u32(smem), 16, 1024);
                const uint64_t dk0 = umma_desc_sw128(smem_u32(smem + Cfg::OFF_R), 16, 1024);
                for (int cid = u_first; cid < n_units; cid += u_step) {
                    const Unit x = unit_at(cid);
                    const int n_kt = x.n_kt;
                    if (n_kt == 0) continue;
                    auto unit_k = [&](int j, int ku) { return base + (j == 0 ? ku : KU + (j - 1) * (KU + 1) + ku); };
                    if (!mbar_wait(q_full, U & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                    for (int j = 0; j < n_kt; j++, T++) {
                        if constexpr (SDB) {
                            // S buffer T % 2 was last read by P V(T - 2) (its P; its S before that).
                            if (T >= 2 &&
                                !mbar_wait(&pv_done[T & 1], ((T - 2) >> 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag))
                                goto done;
                        } else {
                            // S is free once both CTAs' softmax(T - 1) have copied it into registers.
                            if (!mbar_wait(s_empty, (T & 1) ^ 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                        }
                        tc_fence_after();
                        const uint32_t t_sb = SDB ? t_s + (uint32_t)(T & 1) * 128 : t_s;
                        for (int ku = 0; ku < KU; ku++) {
                            const int iu = unit_k(j, ku), u = iu % AP_UNITS;
                            if (!mbar_wait(&r_full[u], (iu / AP_UNITS) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                            const uint64_t db = dk0 + (uint64_t)(u * (AP_UNIT >> 4));
#pragma unroll
                            for (int c = 0; c < 4; c++) {
#pragma unroll
                                for (int kk = 0; kk < 4; kk++)
                                    mma_bf16_pair(t_sb, dq0 + (uint64_t)((4 * ku + c) * (16384 >> 4) + 2 * kk),
                                                  db + (uint64_t)(c * (8192 >> 4) + 2 * kk), idesc_s, (ku | c | kk) != 0);
                            }
                            mma_commit_pair_both(&r_empty[u]);
                        }
                        mma_commit_pair_both(&s_full[SDB ? (T & 1) : 0]);
                    }
                    mma_commit_pair_both(q_empty);  // Q may be replaced once these MMAs are done
                    base += n_kt * (KU + 1);
                    U++;
                }
            } else {
                constexpr uint32_t idesc_o = umma_idesc(256, ATT_DV, 1, /*b_mn_major=*/true);
                const uint64_t dv0 = umma_desc_sw128(smem_u32(smem + Cfg::OFF_R), 16384, 1024);
                for (int cid = u_first; cid < n_units; cid += u_step) {
                    const Unit x = unit_at(cid);
                    const int n_kt = x.n_kt;
                    if (n_kt == 0) continue;
                    auto unit_v = [&](int j) { return base + KU + j * (KU + 1) + (j + 1 < n_kt ? KU : 0); };
                    for (int j = 0; j < n_kt; j++, T++) {
                        const int b = T & 1;
                        if (!mbar_wait(&p_full[b], (T >> 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                        // The first P V of a unit overwrites O: the previous unit's O must have been read.
                        if (j == 0 && U > 0 && !mbar_wait(o_empty, (U - 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag))
                            goto done;
                        tc_fence_after();
                        const int iu = unit_v(j), u = iu % AP_UNITS;
                        if (!mbar_wait(&r_full[u], (iu / AP_UNITS) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                        const uint64_t dv = dv0 + (uint64_t)(u * (AP_UNIT >> 4));
                        // 16 keys per MMA: 8 packed P columns, 16 V rows (2048 bytes per 64-channel chunk).
#pragma unroll
                        for (int kk = 0; kk < AP_BN / 16; kk++)
                            mma_bf16_pair_ts(t_o, (SDB ? t_s + b * 128 : t_p + b * (AP_BN / 2)) + kk * 8,
                                             dv + (uint64_t)(kk * (2048 >> 4)),
                                             idesc_o, (j | kk) != 0);
                        mma_commit_pair_both(&r_empty[u]);
                        mma_commit_pair_both(&pv_done[b]);
                    }
                    base += n_kt * (KU + 1);
                    U++;
                }
            }
        }
    } else if (warp >= 2 && warp < 2 + Cfg::NSW) {
        const int sw = warp - 2;
        const int e = warp & 3;
        const int ch = SPLIT ? (sw >> 2) : 0;    // column half of S / P / O this thread owns
        constexpr int NC = SPLIT ? 64 : 128;     // S columns per thread
        constexpr int OC = SPLIT ? 128 : 256;    // O columns per thread
        const int r = 32 * e + lane;
        const uint32_t lane_off = (uint32_t)(32 * e) << 16;
        const float LOG2E = 1.4426950408889634f;
        float* xmax = reinterpret_cast<float*>(smem + Cfg::OFF_X);  // [slot][half][128]
        float* xsum = xmax + 2 * 2 * 128;                            // [half][128]
        // Arrivals for the MMA issuer go to the even CTA's barriers. What they guard is TMEM (S read,
        // P written, O read), ordered by tcgen05.wait + tcgen05.fence::before_thread_sync.
        auto arrive_even = [&](uint64_t* bar) {
            if (even) mbar_arrive(bar);
            else mbar_arrive_remote(on_even(bar));
        };
        int T = 0, X = 0;
        bool ok = true;
        // The O epilogue of a unit runs after the next unit's first P has been written (so that P does
        // not wait behind it); pend / pu / pl / pT: the unit waiting for it, its row sum, its last tile.
        bool pend = false;
        Unit pu{};
        float pl = 0.f;
        int pT = 0;
        auto finish = [&]() -> bool {
            if (!mbar_wait(&pv_done[pT & 1], (pT >> 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) return false;
            float lt = pl;
            if constexpr (SPLIT) {
                // Both halves' row sums (the same stale max scaled both), through the next handshake.
                xsum[ch * 128 + r] = lt;
                uint64_t* xb = &xpair[e * 2 + (X & 1)];
                mbar_arrive(xb);
                if (!mbar_wait(xb, (X >> 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) return false;
                lt += *reinterpret_cast<volatile float*>(xsum + (ch ^ 1) * 128 + r);
                X++;
            }
            tc_fence_after();
            const float inv = (lt > 0.f) ? 1.f / lt : 0.f;
            const int ptok = pu.q0r + r / G;
            const int head = pu.g * G + r % G;
            bf16_t* orow = prm.out + ((long)(pu.tile.row0 + ptok) * prm.nh + head) * prm.hd + pu.dsplit * ATT_DV + ch * 128;
            const bool live = ptok < pu.tile.len;
            if constexpr (SPLIT) {
                // Every row of the warp in the sequence: 32 x 32 chunks through the warp's staging tile
                // (64-byte swizzle) by TMA store -- one 3-D box [32 channels][G heads][32 / G tokens]
                // is exactly the warp's 32 rows. (Direct per-row stores touched 32 rows per store
                // instruction and held the unit boundary up for ~6k cycles.)
                if (__all_sync(0xffffffffu, live)) {
                    uint8_t* stg = smem + Cfg::OFF_STG + sw * 2048;
                    const uint32_t swz = (uint32_t)((lane >> 1) & 3);
                    const int tok0 = pu.tile.row0 + pu.q0r + (32 * e) / G;
                    tmem_pipelined<32>(t_o + ch * 128 + lane_off, OC / 32, [&](int c, uint32_t(&o)[32]) -> bool {
                        uint32_t pk[16];
#pragma unroll
                        for (int q = 0; q < 16; q++)
                            pk[q] = bf16x2_bits(__uint_as_float(o[2 * q]) * inv, __uint_as_float(o[2 * q + 1]) * inv);
                        if (lane == 0) bulk_wait_read<0>();  // the tile's previous store is read out
                        __syncwarp();
#pragma unroll
                        for (int j = 0; j < 4; j++)
                            *reinterpret_cast<uint4*>(stg + lane * 64 + ((j ^ swz) << 4)) =
                                make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
                        fence_proxy_async();
                        __syncwarp();
                        if (lane == 0) {
                            tma_store_3d(&tmO, stg, pu.dsplit * ATT_DV + ch * 128 + c * 32, pu.g * G, tok0);
                            bulk_commit();
                        }
                        return true;
                    });
                    tc_fence_before();
                    arrive_even(o_empty);
                    return true;
                }
            }
            // 32-byte stores: each instruction writes whole sectors of 32 rows.
            tmem_pipelined<32>(t_o + ch * 128 + lane_off, OC / 32, [&](int c, uint32_t(&o)[32]) -> bool {
                if (live) {
#pragma unroll
                    for (int q = 0; q < 2; q++) {
                        uint32_t pk[8];
#pragma unroll
                        for (int j = 0; j < 8; j++)
                            pk[j] = bf16x2_bits(__uint_as_float(o[16 * q + 2 * j]) * inv, __uint_as_float(o[16 * q + 2 * j + 1]) * inv);
                        st_global_v8(orow + c * 32 + 16 * q, pk);
                    }
                }
                return true;
            });
            // O has been read: the next unit's first P V may overwrite it.
            tc_fence_before();
            arrive_even(o_empty);
            return true;
        };
        for (int cid = u_first; cid < n_units; cid += u_step) {
            const Unit x = unit_at(cid);
            const int n_kt = x.n_kt;
            if (n_kt == 0) continue;
            const AttnTile& tile = x.tile;
            const int tok = x.q0r + r / G;
            const bool row_valid = tok < tile.len;
            // Keys of this row's sequence, relative to the tile's first row.
            int rs = 0, re = tile.len;
            if (prm.seq_start && row_valid) {
                rs = prm.seq_start[tile.row0 + tok] - tile.row0;
                re = rs + prm.seq_len[tile.row0 + tok];
            }
            float m_used = -INFINITY, l = 0.f;
            for (int j = 0; j < n_kt; j++, T++) {
                const int b = T & 1;
                const uint32_t t_sb = SDB ? t_s + (uint32_t)b * 128 : t_s;
                if (!mbar_wait(&s_full[SDB ? b : 0], SDB ? (T >> 1) & 1 : T & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                float sv[NC];
                {
#pragma unroll
                    for (int c = 0; c < NC / 32; c++) {
                        uint32_t s0[32];
                        tmem_ld32(t_sb + ch * 64 + 32 * c + lane_off, s0);
                        tmem_ld_wait();
#pragma unroll
                        for (int q = 0; q < 32; q++) sv[32 * c + q] = __uint_as_float(s0[q]);
                    }
                    if constexpr (!SDB) {
                        tc_fence_before();
                        arrive_even(s_empty);
                    }
                }
                // Valid key columns of this row in this tile, relative to this thread's first column.
                const int kbase = x.k_lo + j * AP_BN + ch * 64;
                int lo_c = max(0, rs - kbase), hi_c = min(NC, re - kbase);
                if (W >= 0 && row_valid) {
                    lo_c = max(lo_c, tok - W - kbase);
                    hi_c = min(hi_c, tok + W + 1 - kbase);
                }
                if (!__all_sync(0xffffffffu, lo_c <= 0 && hi_c >= NC)) {
#pragma unroll
                    for (int c = 0; c < NC; c++) sv[c] = (c >= lo_c && c < hi_c) ? sv[c] : -INFINITY;
                }
                float mx[8];
#pragma unroll
                for (int c = 0; c < 8; c++) mx[c] = sv[c];
#pragma unroll
                for (int c = 8; c < NC; c++) mx[c & 7] = fmaxf(mx[c & 7], sv[c]);
                float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
                if constexpr (SPLIT) {
                    // The row's other half: slots alternate by handshake, so a slot is rewritten only
                    // after the partner has passed the next handshake (and read this one).
                    float* slot = xmax + (X & 1) * 256;
                    slot[ch * 128 + r] = mt;
                    mbar_arrive(&xpair[e * 2 + (X & 1)]);
                    if (!mbar_wait(&xpair[e * 2 + (X & 1)], (X >> 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) {
                        ok = false;
                        break;
                    }
                    mt = fmaxf(mt, *reinterpret_cast<volatile float*>(slot + (ch ^ 1) * 128 + r));
                    X++;
                }
                float factor = 1.f;
                bool need = false;
                if (mt > m_used) {
                    if (m_used == -INFINITY) {
                        m_used = mt;
                    } else if ((mt - m_used) * LOG2E > ATT_RESCALE_LOG2) {
                        factor = ex2_approx((m_used - mt) * LOG2E);
                        m_used = mt;
                        need = true;
                    }
                }
                if (__any_sync(0xffffffffu, need) && j >= 1) {
                    // O must hold every P V up to tile T - 1 before it is rescaled.
                    if (!mbar_wait(&pv_done[(T - 1) & 1], ((T - 1) >> 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll 1
                    for (int c = 0; c < OC / 32; c++) {
                        uint32_t o[32];
                        tmem_ld32(t_o + ch * 128 + c * 32 + lane_off, o);
                        tmem_ld_wait();
#pragma unroll
                        for (int q = 0; q < 32; q++) o[q] = __float_as_uint(__uint_as_float(o[q]) * factor);
                        tmem_st32(t_o + ch * 128 + c * 32 + lane_off, o);
                    }
                    tmem_st_wait();
                }
                l *= factor;
                if constexpr (SDB) {
                    // P goes over S in buffer b: this thread has read its S.
                } else if (T >= 2) {
                    // P buffer b was last read by P V(T - 2) (possibly of the previous unit).
                    if (!mbar_wait(&pv_done[b], ((T - 2) >> 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                }
                // Row sum over the bf16-ROUNDED probabilities that multiply V (weights sum to exactly l).
                const float bias = (m_used == -INFINITY) ? 0.f : -m_used * LOG2E;
                float lsum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int half = 0; half < NC / 64; half++) {
                    uint32_t pk[32];
#pragma unroll
                    for (int q = 0; q < 32; q++) {
                        const float p0 = ex2_approx(fmaf(sv[64 * half + 2 * q], LOG2E, bias));
                        const float p1 = ex2_approx(fmaf(sv[64 * half + 2 * q + 1], LOG2E, bias));
                        pk[q] = bf16x2_bits(p0, p1);
                        lsum[q & 3] += __uint_as_float(pk[q] << 16) + __uint_as_float(pk[q] & 0xffff0000u);
                    }
                    tmem_st32((SDB ? t_sb : t_p + b * (AP_BN / 2)) + 32 * (ch + half) + lane_off, pk);
                }
                l += (lsum[0] + lsum[1]) + (lsum[2] + lsum[3]);
                tmem_st_wait();
                tc_fence_before();
                arrive_even(&p_full[b]);
                if (j == 0 && pend) {
                    pend = false;
                    if (!finish()) {
                        ok = false;
                        break;
                    }
                }
            }
            if (!ok || *abort_flag) break;
            pend = true;
            pu = x;
            pl = l;
            pT = T - 1;
        }
        if (pend && ok && !*abort_flag) finish();
        if constexpr (SPLIT) {
            if (lane == 0) bulk_wait_all();  // the O stores are complete before the CTA ends
            __syncwarp();
        }
    }
done:
    // Every MMA the even CTA issued (into both CTAs' TMEM) has completed before either CTA frees it:
    // each issuing thread waits for its own.
    if (even && (warp == 1 || warp == Cfg::PV_WARP) && lane == 0) {
        uint64_t* d = &drain[warp == 1 ? 0 : 1];
        mma_commit_pair(smem_u32(d));
        mbar_wait(d, 0, EG2_DEV_TIMEOUT_ATTN, nullptr);
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, 512);
    }
}

// ---------------------------------------------------------------------------------------------
// Head 512 on clusters of four CTAs: S = Q K^T once per key tile, O over all 512 channels.
//
// A 512-channel O of 128 rows fills a CTA's TMEM (512 f32 columns), so one CTA pair cannot hold S
// next to it. The four CTAs of a cluster split the work instead of duplicating S:
//   ranks 0, 1  score pair: Q (bf16, TMEM columns [0, 256): brought into the ring by TMA and copied
//               to TMEM with tcgen05.cp) and S over 256 keys (columns [256, 512)); S = Q K^T as
//               M = 256, N = 256 pair MMAs with A read from TMEM (each CTA holds 128 of the 256 keys
//               of K), and the softmax. The P of each 128-key half of a tile is one message: staged
//               per warp in shared memory in the operand layout of the P V MMA and sent with bulk
//               copies over distributed shared memory, with each row's rescale factor and partial
//               row sum.
//   ranks 2, 3  value pair: O in all 512 TMEM columns; per message O += P V as M = 256 pair MMAs, A =
//               the P received in shared memory (three buffers), B = V (each CTA holds 128 of every
//               256 channels); the correction warps rescale O when a row's maximum moved and write
//               O / l at the end.
// Rank 2 + i holds the same 128 query rows as rank i. Per 128 keys each pair's tensor work is 2,048
// cycles (the two 256-channel halves of the CTA-pair kernel each recompute all of S: 3,072 per
// half); P crosses the cluster at 32 KB per CTA per 128 keys.
//
//   warp 0      TMA producer (score pair: Q once per unit, then this CTA's 128 keys of K; value
//               pair: its V channels)
//   warp 1      TMEM allocation; in the even CTA of each pair lane 0 issues that pair's tcgen05 work
//   warps 2..9  score pair: softmax, two threads per row (128 of the 256 columns each, maxima swapped
//               through shared memory as in the head-256 kernel); the threads of column half h stage
//               message 2 t + h of tile t. Value pair: rescale and O / l.
//   warp 10     score pair: lane 0 sends each staged message (two 16 KB chunks of P and 1 KB of
//               factors and sums) once its value buffer is free. Bulk copies queue behind the K tiles'
//               TMA loads on the SM's copy engine; issued by the softmax threads they held the softmax up
//               ~2,300 cycles on every other tile.
// Barriers (the same offsets in all four CTAs; each pair uses its own): the Q / K / V ring (full in
// the pair's even CTA, empty committed to both), s_full / s_empty (S computed / read by both CTAs'
// softmax); in the score CTAs p_empty per value buffer (committed by the value pair's MMAs: the
// buffer's message has been consumed) and staged per column half (the half's last message has landed,
// so its staging may be rewritten: one arrival from the value CTA) and stg_ready per column half (its
// four softmax warps have staged the half's message); in the value CTAs p_full per
// buffer (the bytes of a message), c_done per buffer (both value CTAs' correction threads have
// applied its factors), pv_done per buffer, o_empty (O read out).
// ---------------------------------------------------------------------------------------------
struct AqCfg {
    static constexpr int THREADS = 352;
    static constexpr int P_BYTES = 128 * AP_BN * 2;       // one message's P: 128 keys x this CTA's 128 rows
    static constexpr int X_BYTES = 128 * 8;               // per row: (factor, partial row sum)
    static constexpr int MSG = P_BYTES + X_BYTES;
    // Score CTAs: staging per column half, the Q / K ring, the split softmax's maxima.
    static constexpr int RING = 4;                        // 32 KB units
    static constexpr int OFF_SP = 0;                      // [2] P staging
    static constexpr int OFF_SX = OFF_SP + 2 * P_BYTES;   // [2] (factor, l) staging
    static constexpr int OFF_R = OFF_SX + 2 * X_BYTES;    // ring (1 KB aligned)
    static constexpr int OFF_M = OFF_R + RING * AP_UNIT;  // [2 slots][2 halves][128] floats
    static constexpr int S_END = OFF_M + 2 * 2 * 128 * 4;
    // Value CTAs: three message buffers, the V ring.
    static constexpr int NBUF = 3;
    static constexpr int VRING = 3;
    static constexpr int OFF_VP = 0;
    static constexpr int OFF_VX = OFF_VP + NBUF * P_BYTES;
    static constexpr int OFF_VR = ((OFF_VX + NBUF * X_BYTES + 1023) / 1024) * 1024;
    static constexpr int V_END = OFF_VR + VRING * AP_UNIT;
    static constexpr int OFF_BAR = S_END > V_END ? S_END : V_END;
    // r_full[4] r_empty[4] s_full s_empty p_empty[3] staged[2] stg_ready[2] xpair[8] p_full[3] c_done[3]
    // pv_done[3] o_empty drain
    static constexpr int N_BARS = 2 * RING + 1 + 1 + NBUF + 2 + 2 + 8 + 3 * NBUF + 1 + 1;
    static constexpr int SMEM = 1024 + OFF_BAR + N_BARS * 8 + 16;
};
static_assert(AqCfg::OFF_R % 1024 == 0 && AqCfg::OFF_VR % 1024 == 0 && AqCfg::SMEM <= 227 * 1024,
              "attention quad: shared memory");

__global__ void __launch_bounds__(AqCfg::THREADS, 1)
    attention_quad_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, AttParams prm) {
    using Cfg = AqCfg;
    constexpr int ARRIVALS = 2 * 256;  // the softmax / correction threads of both CTAs of a pair
    constexpr int ST = 2 * AP_BN;      // keys per S tile
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
    uint64_t* r_full = bars;
    uint64_t* r_empty = r_full + Cfg::RING;
    uint64_t* s_full = r_empty + Cfg::RING;
    uint64_t* s_empty = s_full + 1;
    uint64_t* p_empty = s_empty + 1;
    uint64_t* staged = p_empty + Cfg::NBUF;
    uint64_t* stg_ready = staged + 2;
    uint64_t* xpair = stg_ready + 2;
    uint64_t* p_full = xpair + 8;
    uint64_t* c_done = p_full + Cfg::NBUF;
    uint64_t* pv_done = c_done + Cfg::NBUF;
    uint64_t* o_empty = pv_done + Cfg::NBUF;
    uint64_t* drain = o_empty + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::N_BARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool scorer = rank < 2;
    const uint32_t lead = rank & 2u;  // the pair's even CTA
    const bool even = (rank & 1u) == 0;
    const int ring = scorer ? Cfg::RING : Cfg::VRING;
    const int off_ring = scorer ? Cfg::OFF_R : Cfg::OFF_VR;
    const int n_units = prm.n_tiles * prm.nkv;
    const int u_first = (int)(blockIdx.x >> 2), u_step = (int)(gridDim.x >> 2);
    const int G = prm.G, W = prm.window, tqc = prm.tq;
    // A unit: (pair tile, K/V head); n_st S tiles of 256 keys from k_lo, i.e. 2 n_st messages of 128 keys.
    struct Unit {
        AttnTile tile;
        int g, q0r, k_lo, n_st;
    };
    auto unit_at = [&](int cid) {
        Unit x;
        x.tile = prm.tiles[cid / prm.nkv];
        x.g = cid % prm.nkv;
        x.q0r = x.tile.q0 + (int)(rank & 1u) * tqc;
        const int q_last = min(x.tile.q0 + 2 * tqc, x.tile.len) - 1;
        x.k_lo = (W >= 0) ? max(0, x.tile.q0 - W) : 0;
        const int k_hi = (W >= 0) ? min(x.tile.len, q_last + W + 1) : x.tile.len;
        x.n_st = x.tile.len > 0 ? (k_hi - x.k_lo + ST - 1) / ST : 0;
        return x;
    };

    if (threadIdx.x == 0) {
        for (int u = 0; u < Cfg::RING; u++) {
            mbar_init(&r_full[u], 1);
            mbar_init(&r_empty[u], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_empty, ARRIVALS);
        for (int b = 0; b < Cfg::NBUF; b++) {
            mbar_init(&p_empty[b], 1);
            mbar_init(&p_full[b], 1);
            mbar_init(&c_done[b], ARRIVALS);
            mbar_init(&pv_done[b], 1);
        }
        for (int h = 0; h < 2; h++) {
            mbar_init(&staged[h], 1);
            mbar_init(&stg_ready[h], 4);
        }
        for (int x = 0; x < 8; x++) mbar_init(&xpair[x], 64);
        mbar_init(o_empty, ARRIVALS);
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) tmem_alloc_pair(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // A value CTA expects the first message of each buffer before any score CTA can send one.
    if (!scorer && threadIdx.x == 64)
        for (int b = 0; b < Cfg::NBUF; b++) mbar_arrive_expect_tx(&p_full[b], Cfg::MSG);
    cluster_sync();
    grid_dep_launch();
    grid_dep_wait();
    const uint32_t tmem = *tmem_slot;
    auto arrive_lead = [&](uint64_t* bar) {
        if (even) mbar_arrive(bar);
        else mbar_arrive_remote(mapa_shared(smem_u32(bar), lead));
    };

    if (warp == 0) {
        if (lane == 0) {
            int u = 0;
            uint32_t uph = 0;
            auto next_slot = [&](uint8_t*& dst, uint32_t& bar) -> bool {
                if (!mbar_wait(&r_empty[u], uph ^ 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) return false;
                if (even) mbar_arrive_expect_tx(&r_full[u], 2 * AP_UNIT);
                bar = mapa_shared(smem_u32(&r_full[u]), lead);
                dst = smem + off_ring + u * AP_UNIT;
                if (++u == ring) {
                    u = 0;
                    uph ^= 1;
                }
                return true;
            };
            for (int cid = u_first; cid < n_units; cid += u_step) {
                const Unit x = unit_at(cid);
                if (x.n_st == 0) continue;
                uint8_t* dst;
                uint32_t bar;
                if (scorer) {
                    // Q: 4 units of this CTA's 128 rows x 128 channels (2 boxes [G heads x tq tokens x 64 ch]).
                    for (int part = 0; part < 4; part++) {
                        if (!next_slot(dst, bar)) goto done;
                        for (int c = 0; c < 2; c++)
                            tma_load_3d_pair(dst + c * 16384, &tmQ, bar, part * 128 + c * 64, x.g * G, x.tile.row0 + x.q0r);
                    }
                }
                for (int t = 0; t < x.n_st; t++) {
                    const int key0 = x.tile.row0 + x.k_lo + t * ST;
                    if (scorer) {
                        // K of this CTA's 128 keys, channels [128 part, 128 part + 128): 2 boxes [128 keys x 64 ch].
                        for (int part = 0; part < 4; part++) {
                            if (!next_slot(dst, bar)) goto done;
                            for (int c = 0; c < 2; c++)
                                tma_load_3d_pair(dst + c * 16384, &tmK, bar, part * 128 + c * 64, x.g, key0 + AP_BN * (int)(rank & 1u));
                        }
                    } else {
                        // Per message (128 keys): V for this CTA's 128 channels of each 256-channel half.
                        for (int m = 0; m < 2; m++)
                            for (int part = 0; part < 2; part++) {
                                if (!next_slot(dst, bar)) goto done;
                                for (int c = 0; c < 2; c++)
                                    tma_load_3d_pair(dst + c * 16384, &tmV, bar, part * 256 + (int)(rank & 1u) * 128 + c * 64, x.g,
                                                     key0 + AP_BN * m);
                            }
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (even && lane == 0) {
            int iu = 0, Ts = 0, T = 0, U = 0;
            auto wait_slot = [&](int& u) -> bool {
                u = iu % ring;
                const bool ok = mbar_wait(&r_full[u], (iu / ring) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag);
                iu++;
                return ok;
            };
            if (scorer) {
                constexpr uint32_t idesc_s = umma_idesc(256, ST, 1);
                const uint64_t dr0 = umma_desc_sw128(smem_u32(smem + Cfg::OFF_R), 16, 1024);
                const uint32_t t_s = tmem + 256;
                for (int cid = u_first; cid < n_units; cid += u_step) {
                    const Unit x = unit_at(cid);
                    if (x.n_st == 0) continue;
                    // Q into TMEM (channel pairs per column), after the previous unit's S MMAs in issue order.
                    for (int part = 0; part < 4; part++) {
                        int u;
                        if (!wait_slot(u)) goto done;
                        const uint64_t dq = dr0 + (uint64_t)(u * (AP_UNIT >> 4));
#pragma unroll
                        for (int c = 0; c < 2; c++)
#pragma unroll
                            for (int kk = 0; kk < 4; kk++)
                                tmem_cp_pair_128x256b(tmem + (uint32_t)(part * 64 + c * 32 + kk * 8), dq + (uint64_t)(c * (16384 >> 4) + 2 * kk));
                        mma_commit_pair_both(&r_empty[u], 0);
                    }
                    for (int t = 0; t < x.n_st; t++, Ts++) {
                        // S was last read by both CTAs' softmax (Ts - 1).
                        if (Ts >= 1 && !mbar_wait(s_empty, (Ts - 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                        tc_fence_after();
                        for (int part = 0; part < 4; part++) {
                            int u;
                            if (!wait_slot(u)) goto done;
                            const uint64_t db = dr0 + (uint64_t)(u * (AP_UNIT >> 4));
#pragma unroll
                            for (int c = 0; c < 2; c++) {
#pragma unroll
                                for (int kk = 0; kk < 4; kk++)
                                    mma_bf16_pair_ts(t_s, tmem + (uint32_t)(part * 64 + c * 32 + kk * 8),
                                                     db + (uint64_t)(c * (16384 >> 4) + 2 * kk), idesc_s, (part | c | kk) != 0);
                            }
                            mma_commit_pair_both(&r_empty[u], 0);
                        }
                        mma_commit_pair_both(s_full, 0);
                    }
                    U++;
                }
            } else {
                constexpr uint32_t idesc_o = umma_idesc(256, ATT_DV, 1, /*b_mn_major=*/true);
                const uint64_t dv0 = umma_desc_sw128(smem_u32(smem + Cfg::OFF_VR), 16384, 1024);
                const uint64_t dp0 = umma_desc_sw128(smem_u32(smem + Cfg::OFF_VP), 16, 1024);
                for (int cid = u_first; cid < n_units; cid += u_step) {
                    const Unit x = unit_at(cid);
                    if (x.n_st == 0) continue;
                    for (int j = 0; j < 2 * x.n_st; j++, T++) {
                        const int b = T % Cfg::NBUF;
                        // Message T has landed in both value CTAs and its factors are applied to O.
                        if (!mbar_wait(&c_done[b], (T / Cfg::NBUF) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                        // The first P V of a unit overwrites O: the previous unit's O must have been read.
                        if (j == 0 && U > 0 && !mbar_wait(o_empty, (U - 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                        tc_fence_after();
                        const uint64_t dp = dp0 + (uint64_t)(b * (Cfg::P_BYTES >> 4));
                        for (int h = 0; h < 2; h++) {
                            int u;
                            if (!wait_slot(u)) goto done;
                            const uint64_t dv = dv0 + (uint64_t)(u * (AP_UNIT >> 4));
                            // 16 keys per MMA: P chunk kk / 4 (64 keys), 32 bytes into its rows; 16 V rows.
#pragma unroll
                            for (int kk = 0; kk < AP_BN / 16; kk++)
                                mma_bf16_pair(tmem + (uint32_t)(256 * h), dp + (uint64_t)((kk >> 2) * (16384 >> 4) + 2 * (kk & 3)),
                                              dv + (uint64_t)(kk * (2048 >> 4)), idesc_o, (j | kk) != 0);
                            mma_commit_pair_both(&r_empty[u], 2);
                        }
                        mma_commit_pair_both(&pv_done[b], 2);
                        mma_commit_pair_both(&p_empty[b], 0);  // to the score CTAs
                    }
                    U++;
                }
            }
        }
    } else if (warp == 10) {
        if (scorer && lane == 0) {
            int Ts = 0;
            for (int cid = u_first; cid < n_units; cid += u_step) {
                const Unit x = unit_at(cid);
                for (int t = 0; t < x.n_st; t++, Ts++)
                    for (int h = 0; h < 2; h++) {
                        // Message m = 2 Ts + h from staging h into value buffer m % 3 of CTA rank + 2, once the
                        // half has staged it and P V of message m - 3 has completed.
                        const int m = 2 * Ts + h, vb = m % Cfg::NBUF;
                        if (!mbar_wait(&stg_ready[h], Ts & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                        if (m >= Cfg::NBUF && !mbar_wait(&p_empty[vb], (m / Cfg::NBUF - 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag))
                            goto done;
                        const uint32_t peer = rank + 2;
                        const uint32_t pbar = mapa_shared(smem_u32(&p_full[vb]), peer);
                        for (int c = 0; c < 2; c++)
                            bulk_copy_to_peer(mapa_shared(smem_u32(smem + Cfg::OFF_VP + vb * Cfg::P_BYTES + c * 16384), peer),
                                              smem_u32(smem + Cfg::OFF_SP + h * Cfg::P_BYTES + c * 16384), 16384, pbar);
                        bulk_copy_to_peer(mapa_shared(smem_u32(smem + Cfg::OFF_VX + vb * Cfg::X_BYTES), peer),
                                          smem_u32(smem + Cfg::OFF_SX + h * Cfg::X_BYTES), Cfg::X_BYTES, pbar);
                    }
            }
        }
    } else {
        const int e = warp & 3;
        const int ch = (warp - 2) >> 2;  // score pair: S columns [128 ch, +128) (message half ch); value pair: O columns [256 ch, +256)
        const int r = 32 * e + lane;
        const uint32_t lane_off = (uint32_t)(32 * e) << 16;
        const float LOG2E = 1.4426950408889634f;
        int Ts = 0, T = 0, X = 0;
        for (int cid = u_first; cid < n_units; cid += u_step) {
            const Unit x = unit_at(cid);
            if (x.n_st == 0) continue;
            const AttnTile& tile = x.tile;
            const int tok = x.q0r + r / G;
            const int head = x.g * G + r % G;
            const bool row_valid = tok < tile.len;
            bool ok = true;
            if (scorer) {
                int rs = 0, re = tile.len;
                if (prm.seq_start && row_valid) {
                    rs = prm.seq_start[tile.row0 + tok] - tile.row0;
                    re = rs + prm.seq_len[tile.row0 + tok];
                }
                float* xmax = reinterpret_cast<float*>(smem + Cfg::OFF_M);  // [slot][half][128]
                float m_used = -INFINITY, l = 0.f;
                for (int t = 0; t < x.n_st; t++, Ts++) {
                    if (!mbar_wait(s_full, Ts & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    float sv[128];
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        uint32_t s0[32];
                        tmem_ld32(tmem + (uint32_t)(256 + 128 * ch + 32 * c) + lane_off, s0);
                        tmem_ld_wait();
#pragma unroll
                        for (int q = 0; q < 32; q++) sv[32 * c + q] = __uint_as_float(s0[q]);
                    }
                    tc_fence_before();
                    arrive_lead(s_empty);
                    // Valid key columns of this row in this tile, relative to this thread's first column.
                    const int kbase = x.k_lo + t * ST + AP_BN * ch;
                    int lo_c = max(0, rs - kbase), hi_c = min(AP_BN, re - kbase);
                    if (W >= 0 && row_valid) {
                        lo_c = max(lo_c, tok - W - kbase);
                        hi_c = min(hi_c, tok + W + 1 - kbase);
                    }
                    if (!__all_sync(0xffffffffu, lo_c <= 0 && hi_c >= AP_BN)) {
#pragma unroll
                        for (int c = 0; c < AP_BN; c++) sv[c] = (c >= lo_c && c < hi_c) ? sv[c] : -INFINITY;
                    }
                    float mx[8];
#pragma unroll
                    for (int c = 0; c < 8; c++) mx[c] = sv[c];
#pragma unroll
                    for (int c = 8; c < AP_BN; c++) mx[c & 7] = fmaxf(mx[c & 7], sv[c]);
                    float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
                    {
                        // The row's other half (slots alternate by handshake, as in the head-256 kernel).
                        float* slot = xmax + (X & 1) * 256;
                        slot[ch * 128 + r] = mt;
                        mbar_arrive(&xpair[e * 2 + (X & 1)]);
                        if (!mbar_wait(&xpair[e * 2 + (X & 1)], (X >> 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) {
                            ok = false;
                            break;
                        }
                        mt = fmaxf(mt, *reinterpret_cast<volatile float*>(slot + (ch ^ 1) * 128 + r));
                        X++;
                    }
                    float factor = 1.f;
                    if (mt > m_used) {
                        if (m_used == -INFINITY) {
                            m_used = mt;
                        } else if ((mt - m_used) * LOG2E > ATT_RESCALE_LOG2) {
                            factor = ex2_approx((m_used - mt) * LOG2E);
                            m_used = mt;
                        }
                    }
                    l *= factor;
                    // Row sum over the bf16-ROUNDED probabilities that multiply V (weights sum to exactly l).
                    const float bias = (m_used == -INFINITY) ? 0.f : -m_used * LOG2E;
                    float lsum[4] = {0.f, 0.f, 0.f, 0.f};
                    uint32_t pk[64];
#pragma unroll
                    for (int q = 0; q < 64; q++) {
                        const float p0 = ex2_approx(fmaf(sv[2 * q], LOG2E, bias));
                        const float p1 = ex2_approx(fmaf(sv[2 * q + 1], LOG2E, bias));
                        pk[q] = bf16x2_bits(p0, p1);
                        lsum[q & 3] += __uint_as_float(pk[q] << 16) + __uint_as_float(pk[q] & 0xffff0000u);
                    }
                    l += (lsum[0] + lsum[1]) + (lsum[2] + lsum[3]);
                    // Staging ch (message 2 Ts + ch) is free once the half's previous message has landed.
                    if (Ts >= 1 && !mbar_wait(&staged[ch], (Ts - 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) {
                        ok = false;
                        break;
                    }
                    // P row r, keys [64 c, 64 c + 64) of the message: row r of chunk c, 16-byte units swizzled by r % 8.
                    uint8_t* prow = smem + Cfg::OFF_SP + ch * Cfg::P_BYTES + r * 128;
#pragma unroll
                    for (int c = 0; c < 2; c++)
#pragma unroll
                        for (int g = 0; g < 8; g++)
                            *reinterpret_cast<uint4*>(prow + c * 16384 + ((g ^ (r & 7)) << 4)) =
                                make_uint4(pk[32 * c + 4 * g], pk[32 * c + 4 * g + 1], pk[32 * c + 4 * g + 2], pk[32 * c + 4 * g + 3]);
                    // The factor applies to O before the tile's first message; the partial sum is this half's.
                    *reinterpret_cast<float2*>(smem + Cfg::OFF_SX + ch * Cfg::X_BYTES + r * 8) = make_float2(ch == 0 ? factor : 1.f, l);
                    fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&stg_ready[ch]);  // the copy warp sends it
                }
                if (!ok || *abort_flag) break;
            } else {
                float lh0 = 0.f, lh1 = 0.f;  // latest partial row sums of the two column halves
                for (int j = 0; j < 2 * x.n_st; j++, T++) {
                    const int b = T % Cfg::NBUF;
                    if (!mbar_wait(&p_full[b], (T / Cfg::NBUF) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) {
                        ok = false;
                        break;
                    }
                    if (warp == 2 && lane == 0) {
                        // The buffer's next message (T + 3) is sent only after P V(T), which waits for c_done(T).
                        mbar_arrive_expect_tx(&p_full[b], Cfg::MSG);
                        // The sender's staging of column half T % 2 may be rewritten.
                        mbar_arrive_remote(mapa_shared(smem_u32(&staged[T & 1]), rank - 2));
                    }
                    const float2 xv = reinterpret_cast<const float2*>(smem + Cfg::OFF_VX + b * Cfg::X_BYTES)[r];
                    const float factor = xv.x;
                    if (T & 1) lh1 = xv.y;
                    else lh0 = xv.y;
                    if (__any_sync(0xffffffffu, factor != 1.f) && j >= 1) {
                        // O must hold every P V up to message T - 1 before it is rescaled.
                        const int tp = T - 1;
                        if (!mbar_wait(&pv_done[tp % Cfg::NBUF], (tp / Cfg::NBUF) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
#pragma unroll 1
                        for (int c = 0; c < 8; c++) {
                            uint32_t o[32];
                            tmem_ld32(tmem + (uint32_t)(256 * ch + 32 * c) + lane_off, o);
                            tmem_ld_wait();
#pragma unroll
                            for (int q = 0; q < 32; q++) o[q] = __float_as_uint(__uint_as_float(o[q]) * factor);
                            tmem_st32(tmem + (uint32_t)(256 * ch + 32 * c) + lane_off, o);
                        }
                        tmem_st_wait();
                    }
                    tc_fence_before();
                    arrive_lead(&c_done[b]);
                }
                if (!ok || *abort_flag) break;
                // O / l once the unit's last P V has completed; then the next unit may overwrite O.
                const int Tl = T - 1;
                if (!mbar_wait(&pv_done[Tl % Cfg::NBUF], (Tl / Cfg::NBUF) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) break;
                tc_fence_after();
                const float lrow = lh0 + lh1;
                const float inv = (lrow > 0.f) ? 1.f / lrow : 0.f;
                bf16_t* orow = prm.out + ((long)(tile.row0 + tok) * prm.nh + head) * prm.hd + 256 * ch;
                tmem_pipelined<32>(tmem + (uint32_t)(256 * ch) + lane_off, 8, [&](int c, uint32_t(&o)[32]) -> bool {
                    if (row_valid) {
#pragma unroll
                        for (int q = 0; q < 2; q++) {
                            uint32_t pw[8];
#pragma unroll
                            for (int i = 0; i < 8; i++)
                                pw[i] = bf16x2_bits(__uint_as_float(o[16 * q + 2 * i]) * inv, __uint_as_float(o[16 * q + 2 * i + 1]) * inv);
                            st_global_v8(orow + c * 32 + 16 * q, pw);
                        }
                    }
                    return true;
                });
                tc_fence_before();
                arrive_lead(o_empty);
            }
            if (!ok || *abort_flag) break;
        }
    }
done:
    // Every tcgen05 operation a pair's even CTA issued (into both CTAs' TMEM) has completed before
    // either frees it.
    if (even && warp == 1 && lane == 0) {
        mma_commit_pair(smem_u32(drain));
        mbar_wait(drain, 0, EG2_DEV_TIMEOUT_ATTN, nullptr);
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, 512);
    }
}

// ---------------------------------------------------------------------------------------------
// Head 64 (the vision tower: 12 query heads, each with its own K/V head), one CTA per (256 query
// tokens, head): two 128-row query tiles share every K / V tile.
//
// Per 128-key tile and query tile the tensor work is 2 x 256 cycles (S = Q K^T at N = 128, K = 64;
// O += P V at N = 64, K = 128) while the softmax needs ~1,000 cycles of exp2 on the SM's MUFU units,
// so the kernel is softmax-bound: the two query tiles' softmax warp groups run concurrently and the
// MMAs of one run under the other's softmax. TMEM (512 columns): S_h at [128 h, 128 h + 128), P_h
// (packed bf16 pairs) at [256 + 64 h, +64), O_h at [384 + 64 h, +64). S_h(j + 1) is computed as soon
// as softmax_h(j) has copied S_h(j) into registers; P_h(j + 1) is written once P V_h(j) has completed.
// K / V ring of 16 KB units ([128 keys x 64 channels], 128-byte swizzle) in the order K(0), then per
// key tile j K(j + 1) (if any) and V(j).
//
//   warp 0       TMA producer
//   warp 1       TMEM allocation; lane 0 issues S = Q K^T
//   warps 2..5   softmax and O epilogue of query tile 0 (one thread per row); warps 6..9 of tile 1
//   warp 10      lane 0 issues O += P V
// ---------------------------------------------------------------------------------------------
constexpr int A64_UNIT = 16384;
constexpr int A64_RING = 6;
constexpr int A64_PV_WARP = 10;
constexpr int A64_THREADS = 32 * (A64_PV_WARP + 1);
constexpr int A64_OFF_R = 2 * A64_UNIT;
constexpr int A64_OFF_BAR = A64_OFF_R + A64_RING * A64_UNIT;
// q, ring full / empty, s_full[2], s_empty[2], p_full[2], pv_done[2], drain[2]
constexpr int A64_N_BARS = 1 + 2 * A64_RING + 10;
constexpr int A64_SMEM = 1024 + A64_OFF_BAR + A64_N_BARS * 8 + 16;

__global__ void __launch_bounds__(A64_THREADS, 1)
    attention_d64_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, AttParams prm) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + A64_OFF_BAR);
    uint64_t* q_full = bars;
    uint64_t* r_full = bars + 1;
    uint64_t* r_empty = r_full + A64_RING;
    uint64_t* s_full = r_empty + A64_RING;
    uint64_t* s_empty = s_full + 2;
    uint64_t* p_full = s_empty + 2;
    uint64_t* pv_done = p_full + 2;
    uint64_t* drain = pv_done + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + A64_N_BARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int head = (int)blockIdx.y;
    const AttnTile tile = prm.tiles[blockIdx.x];
    const int W = prm.window;
    const int q_last = min(tile.q0 + 256, tile.len) - 1;
    const int k_lo = (W >= 0) ? max(0, tile.q0 - W) : 0;
    const int k_hi = (W >= 0) ? min(tile.len, q_last + W + 1) : tile.len;
    const int n_kt = tile.len > 0 ? (k_hi - k_lo + 127) / 128 : 0;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int u = 0; u < A64_RING; u++) {
            mbar_init(&r_full[u], 1);
            mbar_init(&r_empty[u], 1);
        }
        for (int h = 0; h < 2; h++) {
            mbar_init(&s_full[h], 1);
            mbar_init(&s_empty[h], 128);
            mbar_init(&p_full[h], 128);
            mbar_init(&pv_done[h], 1);
            mbar_init(&drain[h], 1);
        }
        *abort_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t t_s = tmem, t_p = tmem + 256, t_o = tmem + 384;
    // Ring positions of K(j) and V(j).
    auto ring_k = [&](int j) { return j == 0 ? 0 : 2 * j - 1; };
    auto ring_v = [&](int j) { return j + 1 < n_kt ? 2 * j + 2 : 2 * j + 1; };

    if (n_kt == 0) {
        // Padding tile: nothing to do.
    } else if (warp == 0) {
        if (lane == 0) {
            int issued = 0;  // ring loads issued so far (load i: slot i % A64_RING, phase (i / A64_RING) & 1)
            mbar_arrive_expect_tx(q_full, 2 * A64_UNIT);
            for (int h = 0; h < 2; h++)
                tma_load_3d(smem + h * A64_UNIT, &tmQ, q_full, 0, head, tile.row0 + tile.q0 + 128 * h);
            int u = 0;
            uint32_t uph = 0;
            auto load = [&](const CUtensorMap* m, int j) -> bool {
                if (!mbar_wait(&r_empty[u], uph ^ 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) return false;
                mbar_arrive_expect_tx(&r_full[u], A64_UNIT);
                tma_load_3d(smem + A64_OFF_R + u * A64_UNIT, m, &r_full[u], 0, head, tile.row0 + k_lo + 128 * j);
                issued++;
                if (++u == A64_RING) {
                    u = 0;
                    uph ^= 1;
                }
                return true;
            };
            bool ok = load(&tmK, 0);
            for (int j = 0; ok && j < n_kt; j++) {
                if (j + 1 < n_kt) ok = load(&tmK, j + 1);
                if (ok) ok = load(&tmV, j);
            }
            // Every load has landed before the CTA may end (on the error path too).
            mbar_drain(q_full, 0, 200000000ull);
            for (int i = max(0, issued - A64_RING); i < issued; i++)
                mbar_drain(&r_full[i % A64_RING], (uint32_t)((i / A64_RING) & 1), 200000000ull);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_s = umma_idesc(128, 128, 1);
            const uint64_t dk0 = umma_desc_sw128(smem_u32(smem + A64_OFF_R), 16, 1024);
            if (!mbar_wait(q_full, 0, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
            for (int j = 0; j < n_kt; j++) {
                const int iu = ring_k(j), u = iu % A64_RING;
                if (!mbar_wait(&r_full[u], (iu / A64_RING) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                for (int h = 0; h < 2; h++) {
                    // S_h is free once softmax_h(j - 1) has copied it into registers.
                    if (j >= 1 && !mbar_wait(&s_empty[h], (j - 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                    tc_fence_after();
                    const uint64_t dq = umma_desc_sw128(smem_u32(smem + h * A64_UNIT), 16, 1024);
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        mma_bf16(t_s + 128 * h, dq + (uint64_t)(2 * kk), dk0 + (uint64_t)(u * (A64_UNIT >> 4) + 2 * kk),
                                 idesc_s, kk != 0);
                    mma_commit(&s_full[h]);
                }
                mma_commit(&r_empty[u]);
            }
        }
    } else if (warp == A64_PV_WARP) {
        if (lane == 0) {
            constexpr uint32_t idesc_o = umma_idesc(128, 64, 1, /*b_mn_major=*/true);
            const uint64_t dv0 = umma_desc_sw128(smem_u32(smem + A64_OFF_R), 16384, 1024);
            for (int j = 0; j < n_kt; j++) {
                const int iu = ring_v(j), u = iu % A64_RING;
                if (!mbar_wait(&r_full[u], (iu / A64_RING) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                for (int h = 0; h < 2; h++) {
                    if (!mbar_wait(&p_full[h], j & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                    tc_fence_after();
                    // 16 keys per MMA: 8 packed P columns, 16 V rows (2,048 bytes).
#pragma unroll
                    for (int kk = 0; kk < 8; kk++)
                        mma_bf16_ts(t_o + 64 * h, t_p + 64 * h + 8 * kk, dv0 + (uint64_t)(u * (A64_UNIT >> 4) + kk * (2048 >> 4)),
                                    idesc_o, (j | kk) != 0);
                    mma_commit(&pv_done[h]);
                }
                mma_commit(&r_empty[u]);
            }
        }
    } else {
        const int h = (warp - 2) >> 2;
        const int e = warp & 3;
        const int r = 32 * e + lane;
        const uint32_t lane_off = (uint32_t)(32 * e) << 16;
        const int tok = tile.q0 + 128 * h + r;
        const bool row_valid = tok < tile.len;
        int rs = 0, re = tile.len;  // keys of this row's sequence, relative to the tile's first row
        if (prm.seq_start && row_valid) {
            rs = prm.seq_start[tile.row0 + tok] - tile.row0;
            re = rs + prm.seq_len[tile.row0 + tok];
        }
        const float LOG2E = 1.4426950408889634f;
        float m_used = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < n_kt; j++) {
            if (!mbar_wait(&s_full[h], j & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t su[128];
#pragma unroll
            for (int c = 0; c < 4; c++) tmem_ld32(t_s + 128 * h + 32 * c + lane_off, *reinterpret_cast<uint32_t(*)[32]>(su + 32 * c));
            tmem_ld_wait();
            tc_fence_before();
            mbar_arrive(&s_empty[h]);
            float* sv = reinterpret_cast<float*>(su);
            const int kbase = k_lo + 128 * j;
            int lo_c = max(0, rs - kbase), hi_c = min(128, re - kbase);
            if (W >= 0 && row_valid) {
                lo_c = max(lo_c, tok - W - kbase);
                hi_c = min(hi_c, tok + W + 1 - kbase);
            }
            if (!__all_sync(0xffffffffu, lo_c <= 0 && hi_c >= 128)) {
#pragma unroll
                for (int c = 0; c < 128; c++) sv[c] = (c >= lo_c && c < hi_c) ? sv[c] : -INFINITY;
            }
            float mx[8];
#pragma unroll
            for (int c = 0; c < 8; c++) mx[c] = sv[c];
#pragma unroll
            for (int c = 8; c < 128; c++) mx[c & 7] = fmaxf(mx[c & 7], sv[c]);
            const float mt =
                fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
            float factor = 1.f;
            bool need = false;
            if (mt > m_used) {
                if (m_used == -INFINITY) {
                    m_used = mt;
                } else if ((mt - m_used) * LOG2E > ATT_RESCALE_LOG2) {
                    factor = ex2_approx((m_used - mt) * LOG2E);
                    m_used = mt;
                    need = true;
                }
            }
            if (j >= 1) {
                // P V_h(j - 1) has read P_h and added into O_h: both may be rewritten.
                if (!mbar_wait(&pv_done[h], (j - 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
                    for (int c = 0; c < 2; c++) {
                        uint32_t o[32];
                        tmem_ld32(t_o + 64 * h + 32 * c + lane_off, o);
                        tmem_ld_wait();
#pragma unroll
                        for (int q = 0; q < 32; q++) o[q] = __float_as_uint(__uint_as_float(o[q]) * factor);
                        tmem_st32(t_o + 64 * h + 32 * c + lane_off, o);
                    }
                }
            }
            l *= factor;
            // Row sum over the bf16-ROUNDED probabilities that multiply V (weights sum to exactly l).
            const float bias = (m_used == -INFINITY) ? 0.f : -m_used * LOG2E;
            float lsum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int qtr = 0; qtr < 4; qtr++) {
                uint32_t pk[16];
#pragma unroll
                for (int q = 0; q < 16; q++) {
                    const float p0 = ex2_approx(fmaf(sv[32 * qtr + 2 * q], LOG2E, bias));
                    const float p1 = ex2_approx(fmaf(sv[32 * qtr + 2 * q + 1], LOG2E, bias));
                    pk[q] = bf16x2_bits(p0, p1);
                    lsum[q & 3] += __uint_as_float(pk[q] << 16) + __uint_as_float(pk[q] & 0xffff0000u);
                }
                tmem_st16(t_p + 64 * h + 16 * qtr + lane_off, pk);
            }
            l += (lsum[0] + lsum[1]) + (lsum[2] + lsum[3]);
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(&p_full[h]);
        }
        if (ok && mbar_wait(&pv_done[h], (n_kt - 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) {
            tc_fence_after();
            const float inv = (l > 0.f) ? 1.f / l : 0.f;
            bf16_t* orow = prm.out + ((long)(tile.row0 + tok) * prm.nh + head) * 64;
#pragma unroll 1
            for (int c = 0; c < 2; c++) {
                uint32_t o[32];
                tmem_ld32(t_o + 64 * h + 32 * c + lane_off, o);
                tmem_ld_wait();
                if (row_valid) {
#pragma unroll
                    for (int q = 0; q < 2; q++) {
                        uint32_t pk[8];
#pragma unroll
                        for (int i = 0; i < 8; i++)
                            pk[i] = bf16x2_bits(__uint_as_float(o[16 * q + 2 * i]) * inv,
                                                __uint_as_float(o[16 * q + 2 * i + 1]) * inv);
                        st_global_v8(orow + 32 * c + 16 * q, pk);
                    }
                }
            }
        }
    }
done:
    // Every MMA has completed before TMEM is freed: each issuing thread waits for its own.
    if (n_kt > 0 && (warp == 1 || warp == A64_PV_WARP) && lane == 0) {
        uint64_t* d = &drain[warp == 1 ? 0 : 1];
        mma_commit(d);
        mbar_wait(d, 0, EG2_DEV_TIMEOUT_ATTN, nullptr);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

static int launch_d64(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const AttParams& prm,
                      cudaStream_t s) {
    static bool attr_set[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -3;
    if (!attr_set[dev]) {
        if (cudaFuncSetAttribute(attention_d64_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, A64_SMEM) != cudaSuccess)
            return -3;
        attr_set[dev] = true;
    }
    attention_d64_kernel<<<dim3((unsigned)prm.n_tiles, (unsigned)prm.nh, 1), A64_THREADS, A64_SMEM, s>>>(mq, mk, mv, prm);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int attention_tc_tile_tokens(int nh, int nkv, int hd) {
    if (nh <= 0 || nkv <= 0 || nh % nkv) return 0;
    const int G = nh / nkv;
    if (hd == 64) return G == 1 ? 256 : 0;  // two 128-row query tiles of one head
    if ((hd != 256 && hd != 512) || 128 % G) return 0;
    // CTA pairs: one tile covers both CTAs' 128 rows.
    return 256 / G;
}

// As many clusters as can be resident at once (at most one per work unit); each walks its units.
template <int DQK>
static int launch_pair(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mo,
                       const AttParams& prm, cudaStream_t s) {
    using Cfg = ApCfg<DQK>;
    auto kern = attention_pair_kernel<DQK>;
    static int max_clusters[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -3;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute la[2];
    la[0].id = cudaLaunchAttributeClusterDimension;
    la[0].val.clusterDim.x = 2;
    la[0].val.clusterDim.y = 1;
    la[0].val.clusterDim.z = 1;
    la[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    la[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.blockDim = dim3(Cfg::THREADS, 1, 1);
    cfg.dynamicSmemBytes = Cfg::SMEM;
    cfg.stream = s;
    cfg.attrs = la;
    cfg.numAttrs = 1;
    if (!max_clusters[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM) != cudaSuccess) return -3;
        cfg.gridDim = dim3(2 * num_sms(), 1, 1);
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) return -3;
        max_clusters[dev] = n;
    }
    const long units = (long)prm.n_tiles * prm.nkv * prm.nsplit;
    const int clusters = units < max_clusters[dev] ? (int)units : max_clusters[dev];
    cfg.gridDim = dim3((unsigned)(2 * clusters), 1, 1);
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, mq, mk, mv, mo, prm) == cudaSuccess ? 0 : -3;
}

// Head 512: clusters of four (as many as can be resident, at most one per unit), each walking its units.
static int launch_quad(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const AttParams& prm,
                       cudaStream_t s) {
    using Cfg = AqCfg;
    static int max_clusters[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -3;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute la[2];
    la[0].id = cudaLaunchAttributeClusterDimension;
    la[0].val.clusterDim.x = 4;
    la[0].val.clusterDim.y = 1;
    la[0].val.clusterDim.z = 1;
    la[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    la[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.blockDim = dim3(Cfg::THREADS, 1, 1);
    cfg.dynamicSmemBytes = Cfg::SMEM;
    cfg.stream = s;
    cfg.attrs = la;
    cfg.numAttrs = 1;
    if (!max_clusters[dev]) {
        if (cudaFuncSetAttribute(attention_quad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM) != cudaSuccess)
            return -3;
        cfg.gridDim = dim3(4 * num_sms(), 1, 1);
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, attention_quad_kernel, &cfg) != cudaSuccess || n <= 0) return -3;
        max_clusters[dev] = n;
    }
    const long units = (long)prm.n_tiles * prm.nkv;
    const int clusters = units < max_clusters[dev] ? (int)units : max_clusters[dev];
    cfg.gridDim = dim3((unsigned)(4 * clusters), 1, 1);
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, attention_quad_kernel, mq, mk, mv, prm) == cudaSuccess ? 0 : -3;
}

// Head 512 runs on clusters of four for passes of at least ATT512_QUAD_ROWS rows and on the CTA-pair
// kernel (two clusters per query-tile pair, one per 256-channel half of O, each computing all of S)
// below: one 2,208-token document is 35 units, two waves of the 33 resident clusters of four but
// one of the 74 CTA-pair cluster pairs; from ~130 units on the four-CTA kernel's 1.25x shorter key
// tiles win. The regime depends only on the pass's rows, so a sequence gets the same bits in any pass
// of its regime. EG2_ATT512_PAIR=1 keeps every pass on the CTA pairs.
constexpr long ATT512_QUAD_ROWS = 8192;
static bool att512_pair() {
    static const bool v = [] {
        const char* e = getenv("EG2_ATT512_PAIR");
        return e && *e && *e != '0';
    }();
    return v;
}

int attention_tc(const bf16_t* q, const bf16_t* k, const bf16_t* v, bf16_t* out, long rows, const AttnTile* tiles,
                 int n_tiles, int nh, int nkv, int hd, int window, cudaStream_t s, const int* seq_start,
                 const int* seq_len) {
    if (rows <= 0 || n_tiles <= 0) return 0;
    if ((hd != 64 && hd != 256 && hd != 512) || !attention_tc_tile_tokens(nh, nkv, hd)) return -1;
    const int G = nh / nkv;
    if (hd == 64) {
        // q / k / v [rows, heads, 64]: box (64 ch, 1 head, 128 tokens) = 128 rows of 128 B.
        CUtensorMap mq, mk, mv;
        const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
        if (make_tmap_3d(&mq, dt, q, 64, nh, rows, 128, (uint64_t)nh * 128, 64, 1, 128) ||
            make_tmap_3d(&mk, dt, k, 64, nkv, rows, 128, (uint64_t)nkv * 128, 64, 1, 128) ||
            make_tmap_3d(&mv, dt, v, 64, nkv, rows, 128, (uint64_t)nkv * 128, 64, 1, 128))
            return -1;
        AttParams prm{};
        prm.tiles = tiles;
        prm.out = out;
        prm.seq_start = seq_start;
        prm.seq_len = seq_len;
        prm.nh = nh;
        prm.nkv = nkv;
        prm.hd = 64;
        prm.window = window;
        prm.G = 1;
        prm.tq = 256;
        prm.nsplit = 1;
        prm.n_tiles = n_tiles;
        return launch_d64(mq, mk, mv, prm, s);
    }
    const int tq = 128 / G;  // query tokens per CTA (128 MMA rows)
    CUtensorMap mq, mk, mv, mo;
    const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    // q [rows, nh, hd]: box (64 ch, G heads, tq tokens) -> 128 rows of 128 B.
    if (make_tmap_3d(&mq, dt, q, hd, nh, rows, (uint64_t)hd * 2, (uint64_t)nh * hd * 2, 64, G, tq) ||
        make_tmap_3d(&mk, dt, k, hd, nkv, rows, (uint64_t)hd * 2, (uint64_t)nkv * hd * 2, 64, 1, ATT_KBOX) ||
        make_tmap_3d(&mv, dt, v, hd, nkv, rows, (uint64_t)hd * 2, (uint64_t)nkv * hd * 2, 64, 1, AP_BN))
        return -1;
    // out [rows, nh, hd] for the O epilogue's TMA stores (head 256): box (32 ch, G heads, 32 / G tokens)
    // = one warp's 32 rows, 64-byte swizzle.
    if (hd == 256 && make_tmap_3d(&mo, dt, out, hd, nh, rows, (uint64_t)hd * 2, (uint64_t)nh * hd * 2, 32, G, 32 / G,
                                  CU_TENSOR_MAP_SWIZZLE_64B))
        return -1;
    if (hd != 256) mo = mq;  // unused
    AttParams prm;
    prm.tiles = tiles;
    prm.out = out;
    prm.seq_start = seq_start;
    prm.seq_len = seq_len;
    prm.nh = nh;
    prm.nkv = nkv;
    prm.hd = hd;
    prm.window = window;
    prm.G = G;
    prm.tq = tq;
    prm.nsplit = hd / ATT_DV;
    prm.n_tiles = n_tiles;
    prm.q = q;
    prm.rows = rows;
    if (hd == 512 && rows >= ATT512_QUAD_ROWS && !att512_pair()) {
        // K in boxes of 128 keys (a CTA's half of a 256-key S tile).
        CUtensorMap mk2;
        if (make_tmap_3d(&mk2, dt, k, hd, nkv, rows, (uint64_t)hd * 2, (uint64_t)nkv * hd * 2, 64, 1, AP_BN)) return -1;
        prm.nsplit = 1;
        return launch_quad(mq, mk2, mv, prm, s);
    }
    // CTA pairs: clusters of 2 walking the (pair tile, K/V head, 256-channel half of O) units.
    return hd == 256 ? launch_pair<256>(mq, mk, mv, mo, prm, s) : launch_pair<512>(mq, mk, mv, mo, prm, s);
}



}  // namespace eg2

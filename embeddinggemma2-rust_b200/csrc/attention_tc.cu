// Varlen packed flash attention on tcgen05 for the text backbone: bidirectional, scale 1,
// inclusive sliding window (radius `window`) or global, block-diagonal over packed sequences.
//
// Replaces the reference's bf16 flash kernels `flash_attn_d256_packed_bb` and `flash_attn_d512_bb`
// (kernels_sm80.cu:236-416, :474-684; mma.sync) and their launchers (src/gpu/mod.rs:1217-1241,
// :1547-1599); semantics of src/ops.rs:364-444.
//
// One CTA per (query tile, K/V head, output half). A query tile packs the G = nh / nkv query heads
// that share a K/V head into the 128 MMA rows: row r = token (r / G), head (g * G + r % G), so
// each K/V tile loaded serves all G heads. Sliding layers (G = 2) take 64 tokens per tile, global
// layers (G = 4) 32. The output is produced 256 channels at a time: head_dim 512 runs two CTAs per
// tile, each computing the full S = Q K^T and its half of O (TMEM holds 512 fp32 columns, too few
// for S and a 512-wide O together).
//
//   warp 0      TMA: Q once (head_dim / 64 swizzled [128 x 64] boxes), then per 64-key tile the
//               K chunks (ring of 4 x [64 x 64]) and the V tile [64 keys x 256] (VB buffers)
//   warp 1      TMEM owner; lane 0 issues S = Q K^T (M 128, N 64, K 16) and O += P V (M 128,
//               N 256, K 16, P read from TMEM, V read MN-major) and commits. Head 256 keeps Q in
//               TMEM too (one S buffer); head 512 reads Q from shared memory (two S buffers)
//   warps 2..5  softmax: thread = row; (head 256: first copies its Q row into TMEM) reads S from
//               TMEM, masks, online max / sum in the log2 domain, writes P as packed bf16 pairs
//               into P[j % 2] in TMEM; O is rescaled in TMEM only
//               when a row max grows by more than 2^8 (else the stale max is kept, which is exact);
//               at the end O / l is stored as bf16.
#include "common.cuh"
#include "kernels.h"

namespace eg2 {

constexpr int ATT_THREADS = 224;  // warp 0 Q/K loads, 1 MMA, 2..5 softmax, 6 V loads
constexpr int ATT_V_WARP = 6;
constexpr int ATT_BN = 64;       // keys per tile
constexpr int ATT_DV = 256;      // output channels per CTA
// K chunk ring depth (slots of [64 keys x 64 channels]): as deep as shared memory allows.
template <int DQK>
constexpr int att_kst() { return DQK == 256 ? 8 : 4; }
// K chunks per barrier group: one mbarrier wait and one commit per group. The single thread that
// issues the MMAs can only keep a couple of them queued, so every wait / commit between two MMA
// groups leaves the tensor pipe idle; head 256 therefore loads and releases K a whole tile (4
// chunks) at a time, head 512 two chunks at a time.
template <int DQK>
constexpr int att_kgrp() { return DQK == 256 ? 4 : 2; }
constexpr float ATT_RESCALE_LOG2 = 8.f;

template <int DQK, int VB>
struct AttCfg {
    static constexpr int Q_BYTES = (DQK / 64) * 128 * 128;
    static constexpr int K_SLOT = ATT_BN * 128;          // [64 keys x 64 ch] bf16
    static constexpr int V_BYTES = (ATT_DV / 64) * ATT_BN * 128;
    static constexpr int OFF_K = Q_BYTES;
    static constexpr int OFF_V = OFF_K + att_kst<DQK>() * K_SLOT;
    static constexpr int OFF_BAR = OFF_V + VB * V_BYTES;
    static constexpr int SMEM = 1024 + OFF_BAR + 256;
};

struct AttParams {
    const AttnTile* tiles;
    bf16_t* out;
    int nh, nkv, hd, window, G, tq, nsplit;
};

template <int DQK, int VB>
__global__ void __launch_bounds__(ATT_THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, AttParams prm) {
    using Cfg = AttCfg<DQK, VB>;
    constexpr int QCH = DQK / 64;
    // Head 256: Q is copied into TMEM and the S = Q K^T MMAs read it from there (only K comes from
    // shared memory, which is the bandwidth these MMAs are limited by); one S buffer then fits.
    constexpr bool QT = DQK == 256;
    constexpr int NS = QT ? 1 : 2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
    uint64_t* q_full = bars;
    constexpr int KGRP = att_kgrp<DQK>();
    constexpr int NKG = att_kst<DQK>() / KGRP;  // barrier groups in the K ring
    uint64_t* k_full = bars + 1;
    uint64_t* k_empty = k_full + NKG;
    uint64_t* v_full = k_empty + NKG;
    uint64_t* v_empty = v_full + VB;
    uint64_t* s_full = v_empty + VB;
    uint64_t* s_empty = s_full + 2;
    uint64_t* p_full = s_empty + 2;
    uint64_t* pv_done = p_full + 2;
    uint64_t* q_tmem = pv_done + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_tmem + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile_idx = blockIdx.x / (prm.nkv * prm.nsplit);
    const int rem = blockIdx.x % (prm.nkv * prm.nsplit);
    const int g = rem / prm.nsplit, dsplit = rem % prm.nsplit;
    const AttnTile tile = prm.tiles[tile_idx];
    const int G = prm.G, W = prm.window;
    const int q_last = min(tile.q0 + prm.tq, tile.len) - 1;
    const int k_lo = (W >= 0) ? max(0, tile.q0 - W) : 0;
    const int k_hi = (W >= 0) ? min(tile.len, q_last + W + 1) : tile.len;
    const int n_kt = tile.len > 0 ? (k_hi - k_lo + ATT_BN - 1) / ATT_BN : 0;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < NKG; s++) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
        }
        for (int s = 0; s < VB; s++) {
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        for (int s = 0; s < 2; s++) {
            mbar_init(&s_full[s], 1);
            mbar_init(&s_empty[s], 128);
            mbar_init(&p_full[s], 128);
            mbar_init(&pv_done[s], 1);
        }
        mbar_init(q_tmem, 128);
        *abort_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // TMEM columns. Q in TMEM (head 256): S [0, 64) single-buffered, P [64, 128), Q [128, 256),
    // O [256, 512). Q in shared memory (head 512): S[0..1] [0, 128), P [128, 192), O [256, 512).
    // P holds packed bf16 pairs: 32 columns per 64-key tile, two tiles.
    const uint32_t t_s = tmem;
    const uint32_t t_p = tmem + (QT ? 64 : 128);
    const uint32_t t_q = tmem + 128;
    const uint32_t t_o = tmem + 256;

    if (n_kt == 0) goto done;

    if (warp == 0) {
        // K producer (with Q first). K and V have producers of their own so that a wait for a free
        // V buffer never holds back the K loads the next S = Q K^T needs.
        if (lane == 0) {
            // Q: the G heads of K/V head g for tokens [q0, q0 + tq), 128 rows of 64 channels per box.
            mbar_arrive_expect_tx(q_full, Cfg::Q_BYTES);
            for (int c = 0; c < QCH; c++)
                tma_load_3d(smem + c * 128 * 128, &tmQ, q_full, c * 64, g * G, tile.row0 + tile.q0);
            int kg = 0;
            uint32_t kph = 0;
            for (int j = 0; j < n_kt; j++) {
                const int key0 = tile.row0 + k_lo + j * ATT_BN;
                for (int c0 = 0; c0 < QCH; c0 += KGRP) {
                    if (!mbar_wait(&k_empty[kg], kph ^ 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                    mbar_arrive_expect_tx(&k_full[kg], KGRP * Cfg::K_SLOT);
                    for (int cc = 0; cc < KGRP; cc++)
                        tma_load_3d(smem + Cfg::OFF_K + (kg * KGRP + cc) * Cfg::K_SLOT, &tmK, &k_full[kg], (c0 + cc) * 64, g, key0);
                    if (++kg == NKG) {
                        kg = 0;
                        kph ^= 1;
                    }
                }
            }
        }
    } else if (warp == ATT_V_WARP) {
        if (lane == 0) {
            int vs = 0;
            uint32_t vph = 0;
            for (int j = 0; j < n_kt; j++) {
                const int key0 = tile.row0 + k_lo + j * ATT_BN;
                if (!mbar_wait(&v_empty[vs], vph ^ 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                mbar_arrive_expect_tx(&v_full[vs], Cfg::V_BYTES);
                for (int c = 0; c < ATT_DV / 64; c++)
                    tma_load_3d(smem + Cfg::OFF_V + vs * Cfg::V_BYTES + c * ATT_BN * 128, &tmV, &v_full[vs],
                                dsplit * ATT_DV + c * 64, g, key0);
                if (++vs == VB) {
                    vs = 0;
                    vph ^= 1;
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_s = umma_idesc(128, ATT_BN, 1);
            constexpr uint32_t idesc_o = umma_idesc(128, ATT_DV, 1, /*b_mn_major=*/true);
            // Descriptors are built once; moving within a tile only adds (byte offset >> 4) to the
            // start-address field. A single thread issues every MMA, so anything between two
            // tcgen05.mma instructions is issue latency the tensor pipe waits for.
            const uint64_t dq0 = umma_desc_sw128(smem_u32(smem), 16, 1024);
            const uint64_t dk0 = umma_desc_sw128(smem_u32(smem + Cfg::OFF_K), 16, 1024);
            const uint64_t dv0 = umma_desc_sw128(smem_u32(smem + Cfg::OFF_V), ATT_BN * 128, 1024);
            int kg = 0, vs = 0;
            uint32_t kph = 0, vph = 0;
            if (!mbar_wait(QT ? q_tmem : q_full, 0, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
            // S[j % 2] = Q K_j^T over head_dim in 64-channel chunks.
            auto issue_qk = [&](int j) -> bool {
                const int sb = j % NS;
                const uint32_t ts = t_s + sb * ATT_BN;
                if (!mbar_wait(&s_empty[sb], ((j / NS) & 1) ^ 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) return false;
                tc_fence_after();
                for (int c0 = 0; c0 < QCH; c0 += KGRP) {
                    // K arrives by TMA (async proxy, like the MMA's reads): the barrier wait is enough.
                    if (!mbar_wait(&k_full[kg], kph, EG2_DEV_TIMEOUT_ATTN, abort_flag)) return false;
#pragma unroll
                    for (int cc = 0; cc < KGRP; cc++) {
                        const int c = c0 + cc;
                        const uint64_t db = dk0 + (uint64_t)((kg * KGRP + cc) * (Cfg::K_SLOT >> 4));
                        if constexpr (QT) {
                            // A = Q from TMEM: 16 channels = 8 packed columns per MMA.
                            const uint32_t ta = t_q + c * 32;
                            mma_bf16_ts(ts, ta, db, idesc_s, c != 0);
#pragma unroll
                            for (int kk = 1; kk < 4; kk++) mma_bf16_ts(ts, ta + 8 * kk, db + 2 * kk, idesc_s, 1);
                        } else {
                            const uint64_t da = dq0 + (uint64_t)(c * (128 * 128 >> 4));
                            mma_bf16(ts, da, db, idesc_s, c != 0);
#pragma unroll
                            for (int kk = 1; kk < 4; kk++) mma_bf16(ts, da + 2 * kk, db + 2 * kk, idesc_s, 1);
                        }
                    }
                    mma_commit(&k_empty[kg]);
                    if (++kg == NKG) {
                        kg = 0;
                        kph ^= 1;
                    }
                }
                mma_commit(&s_full[sb]);
                return true;
            };
            if (!issue_qk(0)) goto done;
            for (int j = 0; j < n_kt; j++) {
                if (j + 1 < n_kt && !issue_qk(j + 1)) goto done;
                const int pb = j & 1;
                if (!mbar_wait(&p_full[pb], (j >> 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                if (!mbar_wait(&v_full[vs], vph, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                tc_fence_after();
                const uint64_t dv = dv0 + (uint64_t)(vs * (Cfg::V_BYTES >> 4));
                const uint32_t tp = t_p + pb * (ATT_BN / 2);
                // 16 keys per MMA = 8 packed P columns and 16 V rows (2048 bytes).
                mma_bf16_ts(t_o, tp, dv, idesc_o, j != 0);
#pragma unroll
                for (int kk = 1; kk < ATT_BN / 16; kk++) mma_bf16_ts(t_o, tp + kk * 8, dv + kk * (2048 >> 4), idesc_o, 1);
                mma_commit(&v_empty[vs]);
                mma_commit(&pv_done[pb]);
                if (++vs == VB) {
                    vs = 0;
                    vph ^= 1;
                }
            }
        }
    } else {
        // Softmax / epilogue warps: row r = 32 * (warp % 4) + lane of the 128-row tile.
        const int e = warp & 3;
        const int r = 32 * e + lane;
        const int tok = tile.q0 + r / G;  // position within the sequence
        const bool row_valid = tok < tile.len;
        const uint32_t lane_off = (uint32_t)(32 * e) << 16;
        const float LOG2E = 1.4426950408889634f;
        float m_used = -INFINITY, l = 0.f;
        if constexpr (QT) {
            // Q row r into TMEM columns [t_q, t_q + 128): un-swizzle the row from the four 128-byte
            // swizzled TMA boxes; bf16 pairs are already packed the way the A operand wants them.
            if (!mbar_wait(q_full, 0, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
#pragma unroll 1
            for (int c = 0; c < QCH; c++) {
                uint32_t qv[32];
                const uint8_t* rowp = smem + c * 128 * 128 + r * 128;
#pragma unroll
                for (int piece = 0; piece < 8; piece++) {
                    const uint4 u = *reinterpret_cast<const uint4*>(rowp + ((piece ^ (r & 7)) << 4));
                    qv[4 * piece] = u.x, qv[4 * piece + 1] = u.y, qv[4 * piece + 2] = u.z, qv[4 * piece + 3] = u.w;
                }
                tmem_st32(t_q + c * 32 + lane_off, qv);
            }
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(q_tmem);
        }
        for (int j = 0; j < n_kt; j++) {
            const int sb = j % NS, pb = j & 1;
            if (!mbar_wait(&s_full[sb], (j / NS) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) break;
            tc_fence_after();
            uint32_t s0[32], s1[32];
            tmem_ld32(t_s + sb * ATT_BN + lane_off, s0);
            tmem_ld32(t_s + sb * ATT_BN + 32 + lane_off, s1);
            tmem_ld_wait();
            tc_fence_before();
            mbar_arrive(&s_empty[sb]);
            // Valid key columns of this row in this tile: [lo_c, hi_c). Interior tiles (every row of
            // the warp fully valid) skip the masking pass.
            const int kbase = k_lo + j * ATT_BN;  // key position of column 0 within the sequence
            int lo_c = 0, hi_c = min(ATT_BN, tile.len - kbase);
            if (W >= 0 && row_valid) {
                lo_c = max(lo_c, tok - W - kbase);
                hi_c = min(hi_c, tok + W + 1 - kbase);
            }
            float sv[64];
#pragma unroll
            for (int c = 0; c < 32; c++) {
                sv[c] = __uint_as_float(s0[c]);
                sv[32 + c] = __uint_as_float(s1[c]);
            }
            if (!__all_sync(0xffffffffu, lo_c <= 0 && hi_c >= ATT_BN)) {
#pragma unroll
                for (int c = 0; c < 64; c++) sv[c] = (c >= lo_c && c < hi_c) ? sv[c] : -INFINITY;
            }
            // Row max as 8 independent chains (a single warp per SM sub-partition: no other warp hides
            // the latency of a 64-long dependent chain).
            float mx[8];
#pragma unroll
            for (int c = 0; c < 8; c++) mx[c] = sv[c];
#pragma unroll
            for (int c = 8; c < 64; c++) mx[c & 7] = fmaxf(mx[c & 7], sv[c]);
            const float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
            // Reference max (raw logit units): keep the stale one unless the new max exceeds it by
            // 2^8 in probability, so O is rescaled only rarely (the result is exact either way).
            float factor = 1.f;
            bool need = false;
            if (mt > m_used) {
                if (m_used == -INFINITY) {
                    m_used = mt;  // O rows so far are exactly 0 (all earlier P were 0)
                } else if ((mt - m_used) * LOG2E > ATT_RESCALE_LOG2) {
                    factor = ex2_approx((m_used - mt) * LOG2E);
                    m_used = mt;
                    need = true;
                }
            }
            // P buffer reuse: PV(j - 2) must be done. Rescaling O also needs PV(j - 1) done.
            if (j >= 2) {
                if (!mbar_wait(&pv_done[pb], ((j - 2) >> 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) break;
                tc_fence_after();
            }
            const bool warp_need = __any_sync(0xffffffffu, need);
            if (warp_need && j >= 1) {
                if (!mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) break;
                tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < ATT_DV / 32; c++) {
                    uint32_t o[32];
                    tmem_ld32(t_o + c * 32 + lane_off, o);
                    tmem_ld_wait();
#pragma unroll
                    for (int q = 0; q < 32; q++) o[q] = __float_as_uint(__uint_as_float(o[q]) * factor);
                    tmem_st32(t_o + c * 32 + lane_off, o);
                }
                tmem_st_wait();
            }
            l *= factor;
            // p = 2^((s - m_used) log2 e): one FFMA + one MUFU op per element; masked entries are
            // -inf and give 0 (a row with no valid key yet has m_used = -inf: bias 0 keeps it 0).
            // Stored as packed bf16 pairs into P[j % 2] in TMEM (lane = row, column c holds keys 2c
            // and 2c + 1: the A-operand layout of the P V product). The row sum adds the ROUNDED
            // values, so the weights that multiply V sum to exactly l: with few keys an unrounded sum
            // would scale the whole output row by up to 2^-9.
            const float bias = (m_used == -INFINITY) ? 0.f : -m_used * LOG2E;
            float lsum[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t pk[32];
#pragma unroll
            for (int q = 0; q < 32; q++) {
                const float p0 = ex2_approx(fmaf(sv[2 * q], LOG2E, bias));
                const float p1 = ex2_approx(fmaf(sv[2 * q + 1], LOG2E, bias));
                pk[q] = bf16x2_bits(p0, p1);
                lsum[q & 3] += __uint_as_float(pk[q] << 16) + __uint_as_float(pk[q] & 0xffff0000u);
            }
            l += (lsum[0] + lsum[1]) + (lsum[2] + lsum[3]);
            tmem_st32(t_p + pb * (ATT_BN / 2) + lane_off, pk);
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(&p_full[pb]);
        }
        // Epilogue: O / l for this row's 256 channels.
        if (!*abort_flag && mbar_wait(&pv_done[(n_kt - 1) & 1], ((n_kt - 1) >> 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) {
            tc_fence_after();
            const float inv = (l > 0.f) ? 1.f / l : 0.f;
            const int head = g * G + r % G;
            bf16_t* orow = prm.out + ((long)(tile.row0 + tok) * prm.nh + head) * prm.hd + dsplit * ATT_DV;
#pragma unroll 1
            for (int c = 0; c < ATT_DV / 32; c++) {
                uint32_t o[32];
                tmem_ld32(t_o + c * 32 + lane_off, o);
                tmem_ld_wait();
                if (row_valid) {
                    uint4* d = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        d[q] = make_uint4(pack_bf16x2(__uint_as_float(o[8 * q + 0]) * inv, __uint_as_float(o[8 * q + 1]) * inv),
                                          pack_bf16x2(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv),
                                          pack_bf16x2(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv),
                                          pack_bf16x2(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv));
                }
            }
        }
    }
done:
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------------------------------------
// Head 256: CTA pairs (cta_group::2) over 128-key tiles.
//
// A 2-CTA cluster takes two adjacent query tiles of one sequence and K/V head (128 MMA rows each)
// and runs every MMA as one M = 256 tcgen05.mma issued by the even CTA: S = Q K^T at N = 128 keys
// (each CTA holds 64 of them) and O += P V at N = 256 channels (each CTA holds V for 128 of them).
// Each CTA therefore loads and feeds the tensor cores half of every K / V tile, which halves the
// shared-memory traffic per FLOP of a single-CTA kernel (there: 320 KB per 128-key tile against
// 128 B/cycle of shared memory for 2,048 tensor cycles; here 192 KB). Keys span the union of both
// tiles' windows; each row masks its own.
//
// TMEM per CTA: S [0, 128), P[0] [128, 192), P[1] [192, 256) (packed bf16), O [256, 512). Per CTA
// shared memory: Q (64 KB) and a ring of five 32 KB units, consumed in order K(j + 1), V(j); a K unit
// is 64 keys x 256 channels, a V unit 128 keys x 128 channels. The even CTA's barriers collect both
// CTAs' TMA bytes (q_full, r_full) and both CTAs' softmax arrivals (s_empty, p_full: 256); MMA
// completion is committed to the barriers of both CTAs (r_empty, s_full, pv_done).
//
//   warp 0      TMA producer (this CTA's Q and its half of every unit)
//   warp 1      TMEM allocation (both CTAs); in the even CTA lane 0 issues the S = Q K^T MMAs
//   warps 2..5  softmax, one thread per row of this CTA's 128 rows; O / l epilogue
//   warp 6      in the even CTA lane 0 issues the O += P V MMAs
// Two issuing threads: tcgen05.mma issue blocks once a couple of MMAs are queued, so one thread
// leaves the tensor pipe idle during each of its waits and commits; with S and P V on different
// threads (disjoint TMEM, per-thread commit tracking) one feeds the pipe while the other waits.
// ---------------------------------------------------------------------------------------------
constexpr int AP_THREADS = 224;
constexpr int AP_BN = 128;
constexpr int AP_UNITS = 5;
constexpr int AP_UNIT = 32768;
struct ApCfg {
    static constexpr int Q_BYTES = 4 * 128 * 128;
    static constexpr int OFF_R = Q_BYTES;
    static constexpr int OFF_BAR = OFF_R + AP_UNITS * AP_UNIT;
    static constexpr int N_BARS = 1 + 2 * AP_UNITS + 2 + 4 + 2;  // q, ring, s full/empty, p[2], pv[2], drain[2]
    static constexpr int SMEM = 1024 + OFF_BAR + N_BARS * 8 + 16;
};
static_assert(ApCfg::SMEM <= 227 * 1024, "attention pair: shared memory");

__global__ void __launch_bounds__(AP_THREADS, 1)
    attention_pair_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, AttParams prm) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + ApCfg::OFF_BAR);
    uint64_t* q_full = bars;
    uint64_t* r_full = bars + 1;
    uint64_t* r_empty = r_full + AP_UNITS;
    uint64_t* s_full = r_empty + AP_UNITS;
    uint64_t* s_empty = s_full + 1;
    uint64_t* p_full = s_empty + 1;
    uint64_t* pv_done = p_full + 2;
    uint64_t* drain = pv_done + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + ApCfg::N_BARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool even = rank == 0;
    const int cid = (int)(blockIdx.x >> 1);
    const int tile_idx = cid / prm.nkv;
    const int g = cid % prm.nkv;
    const AttnTile tile = prm.tiles[tile_idx];
    const int G = prm.G, W = prm.window, tqc = prm.tq;
    const int q0r = tile.q0 + (int)rank * tqc;  // this CTA's first query token
    const int q_last = min(tile.q0 + 2 * tqc, tile.len) - 1;
    const int k_lo = (W >= 0) ? max(0, tile.q0 - W) : 0;
    const int k_hi = (W >= 0) ? min(tile.len, q_last + W + 1) : tile.len;
    const int n_kt = tile.len > 0 ? (k_hi - k_lo + AP_BN - 1) / AP_BN : 0;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int u = 0; u < AP_UNITS; u++) {
            mbar_init(&r_full[u], 1);
            mbar_init(&r_empty[u], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_empty, 256);
        for (int b = 0; b < 2; b++) {
            mbar_init(&p_full[b], 256);
            mbar_init(&pv_done[b], 1);
        }
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
    const uint32_t tmem = *tmem_slot;
    const uint32_t t_s = tmem;
    const uint32_t t_p = tmem + 128;
    const uint32_t t_o = tmem + 256;
    auto on_even = [&](uint64_t* b) { return mapa_shared(smem_u32(b), 0); };

    if (n_kt == 0) goto done;

    if (warp == 0) {
        if (lane == 0) {
            if (even) mbar_arrive_expect_tx(q_full, 2 * ApCfg::Q_BYTES);
            const uint32_t qbar = on_even(q_full);
            for (int c = 0; c < 4; c++)
                tma_load_3d_pair(smem + c * 128 * 128, &tmQ, qbar, c * 64, g * G, tile.row0 + q0r);
            int u = 0;
            uint32_t uph = 0;
            // K unit of key tile jt: this CTA's 64 keys, 4 boxes of [64 keys x 64 channels]. V unit: all
            // 128 keys for this CTA's 128 channels, 2 boxes of [128 keys x 64 channels].
            auto load_unit = [&](bool is_k, int jt) -> bool {
                if (!mbar_wait(&r_empty[u], uph ^ 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) return false;
                if (even) mbar_arrive_expect_tx(&r_full[u], 2 * AP_UNIT);
                const uint32_t bar = on_even(&r_full[u]);
                uint8_t* dst = smem + ApCfg::OFF_R + u * AP_UNIT;
                const int key0 = tile.row0 + k_lo + jt * AP_BN;
                if (is_k) {
                    for (int c = 0; c < 4; c++) tma_load_3d_pair(dst + c * 8192, &tmK, bar, c * 64, g, key0 + 64 * (int)rank);
                } else {
                    for (int c = 0; c < 2; c++) tma_load_3d_pair(dst + c * 16384, &tmV, bar, (2 * (int)rank + c) * 64, g, key0);
                }
                if (++u == AP_UNITS) {
                    u = 0;
                    uph ^= 1;
                }
                return true;
            };
            if (!load_unit(true, 0)) goto done;
            for (int j = 0; j < n_kt; j++) {
                if (j + 1 < n_kt && !load_unit(true, j + 1)) goto done;
                if (!load_unit(false, j)) goto done;
            }
        }
    } else if (warp == 1 || warp == 6) {
        if (even && lane == 0) {
            // Ring unit of K(j) / V(j): the producer's order is K(0), then per tile j K(j + 1) (if
            // any) and V(j).
            auto unit_k = [&](int j) { return j == 0 ? 0 : 2 * j - 1; };
            auto unit_v = [&](int j) { return j + 1 < n_kt ? 2 * j + 2 : 2 * j + 1; };
            if (warp == 1) {
                constexpr uint32_t idesc_s = umma_idesc(256, AP_BN, 1);
                const uint64_t dq0 = umma_desc_sw128(smem_u32(smem), 16, 1024);
                const uint64_t dk0 = umma_desc_sw128(smem_u32(smem + ApCfg::OFF_R), 16, 1024);
                if (!mbar_wait(q_full, 0, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                for (int j = 0; j < n_kt; j++) {
                    // S is free once both CTAs' softmax(j - 1) have copied it into registers.
                    if (!mbar_wait(s_empty, (j & 1) ^ 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                    tc_fence_after();
                    const int iu = unit_k(j), u = iu % AP_UNITS;
                    if (!mbar_wait(&r_full[u], (iu / AP_UNITS) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                    const uint64_t db = dk0 + (uint64_t)(u * (AP_UNIT >> 4));
#pragma unroll
                    for (int c = 0; c < 4; c++) {
#pragma unroll
                        for (int kk = 0; kk < 4; kk++)
                            mma_bf16_pair(t_s, dq0 + (uint64_t)(c * (16384 >> 4) + 2 * kk),
                                          db + (uint64_t)(c * (8192 >> 4) + 2 * kk), idesc_s, (c | kk) != 0);
                    }
                    mma_commit_pair_both(&r_empty[u]);
                    mma_commit_pair_both(s_full);
                }
            } else {
                constexpr uint32_t idesc_o = umma_idesc(256, ATT_DV, 1, /*b_mn_major=*/true);
                const uint64_t dv0 = umma_desc_sw128(smem_u32(smem + ApCfg::OFF_R), 16384, 1024);
                for (int j = 0; j < n_kt; j++) {
                    const int b = j & 1;
                    if (!mbar_wait(&p_full[b], (j >> 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                    tc_fence_after();
                    const int iu = unit_v(j), u = iu % AP_UNITS;
                    if (!mbar_wait(&r_full[u], (iu / AP_UNITS) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) goto done;
                    const uint64_t dv = dv0 + (uint64_t)(u * (AP_UNIT >> 4));
                    // 16 keys per MMA: 8 packed P columns, 16 V rows (2048 bytes per 64-channel chunk).
#pragma unroll
                    for (int kk = 0; kk < AP_BN / 16; kk++)
                        mma_bf16_pair_ts(t_o, t_p + b * (AP_BN / 2) + kk * 8, dv + (uint64_t)(kk * (2048 >> 4)), idesc_o,
                                         (j | kk) != 0);
                    mma_commit_pair_both(&r_empty[u]);
                    mma_commit_pair_both(&pv_done[b]);
                }
            }
        }
    } else {
        const int e = warp & 3;
        const int r = 32 * e + lane;
        const int tok = q0r + r / G;
        const bool row_valid = tok < tile.len;
        const uint32_t lane_off = (uint32_t)(32 * e) << 16;
        const float LOG2E = 1.4426950408889634f;
        // Arrivals for the MMA issuer go to the even CTA's barriers. What they guard is TMEM (S read,
        // P written), ordered by tcgen05.wait + tcgen05.fence::before_thread_sync.
        auto arrive_even = [&](uint64_t* bar) {
            if (even) mbar_arrive(bar);
            else mbar_arrive_remote(on_even(bar));
        };
        float m_used = -INFINITY, l = 0.f;
        for (int j = 0; j < n_kt; j++) {
            const int b = j & 1;
            if (!mbar_wait(s_full, j & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) break;
            tc_fence_after();
            float sv[AP_BN];
            {
                uint32_t s0[32], s1[32], s2[32], s3[32];
                tmem_ld32(t_s + lane_off, s0);
                tmem_ld32(t_s + 32 + lane_off, s1);
                tmem_ld32(t_s + 64 + lane_off, s2);
                tmem_ld32(t_s + 96 + lane_off, s3);
                tmem_ld_wait();
                tc_fence_before();
                arrive_even(s_empty);
#pragma unroll
                for (int c = 0; c < 32; c++) {
                    sv[c] = __uint_as_float(s0[c]);
                    sv[32 + c] = __uint_as_float(s1[c]);
                    sv[64 + c] = __uint_as_float(s2[c]);
                    sv[96 + c] = __uint_as_float(s3[c]);
                }
            }
            const int kbase = k_lo + j * AP_BN;
            int lo_c = 0, hi_c = min(AP_BN, tile.len - kbase);
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
            const float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
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
                // O must hold every P V up to tile j - 1 before it is rescaled.
                if (!mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) break;
                tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < ATT_DV / 32; c++) {
                    uint32_t o[32];
                    tmem_ld32(t_o + c * 32 + lane_off, o);
                    tmem_ld_wait();
#pragma unroll
                    for (int q = 0; q < 32; q++) o[q] = __float_as_uint(__uint_as_float(o[q]) * factor);
                    tmem_st32(t_o + c * 32 + lane_off, o);
                }
                tmem_st_wait();
            }
            l *= factor;
            // P buffer b was last read by P V(j - 2).
            if (j >= 2) {
                if (!mbar_wait(&pv_done[b], ((j - 2) >> 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) break;
                tc_fence_after();
            }
            // Row sum over the bf16-ROUNDED probabilities that multiply V (weights sum to exactly l).
            const float bias = (m_used == -INFINITY) ? 0.f : -m_used * LOG2E;
            float lsum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int half = 0; half < 2; half++) {
                uint32_t pk[32];
#pragma unroll
                for (int q = 0; q < 32; q++) {
                    const float p0 = ex2_approx(fmaf(sv[64 * half + 2 * q], LOG2E, bias));
                    const float p1 = ex2_approx(fmaf(sv[64 * half + 2 * q + 1], LOG2E, bias));
                    pk[q] = bf16x2_bits(p0, p1);
                    lsum[q & 3] += __uint_as_float(pk[q] << 16) + __uint_as_float(pk[q] & 0xffff0000u);
                }
                tmem_st32(t_p + b * (AP_BN / 2) + 32 * half + lane_off, pk);
            }
            l += (lsum[0] + lsum[1]) + (lsum[2] + lsum[3]);
            tmem_st_wait();
            tc_fence_before();
            arrive_even(&p_full[b]);
        }
        if (!*abort_flag &&
            mbar_wait(&pv_done[(n_kt - 1) & 1], ((n_kt - 1) >> 1) & 1, EG2_DEV_TIMEOUT_ATTN, abort_flag)) {
            tc_fence_after();
            const float inv = (l > 0.f) ? 1.f / l : 0.f;
            const int head = g * G + r % G;
            bf16_t* orow = prm.out + ((long)(tile.row0 + tok) * prm.nh + head) * prm.hd;
#pragma unroll 1
            for (int c = 0; c < ATT_DV / 32; c++) {
                uint32_t o[32];
                tmem_ld32(t_o + c * 32 + lane_off, o);
                tmem_ld_wait();
                if (row_valid) {
                    uint4* d = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        d[q] = make_uint4(pack_bf16x2(__uint_as_float(o[8 * q + 0]) * inv, __uint_as_float(o[8 * q + 1]) * inv),
                                          pack_bf16x2(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv),
                                          pack_bf16x2(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv),
                                          pack_bf16x2(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv));
                }
            }
        }
    }
done:
    // Every MMA the even CTA issued (into both CTAs' TMEM) has completed before either CTA frees it:
    // each issuing thread waits for its own.
    if (even && (warp == 1 || warp == 6) && lane == 0) {
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

int attention_tc_tile_tokens(int nh, int nkv, int hd) {
    if (nkv <= 0 || nh % nkv) return 0;
    const int G = nh / nkv;
    if (128 % G) return 0;
    // Head 256 runs CTA pairs: one tile covers both CTAs' 128 rows.
    return (hd == 256 ? 256 : 128) / G;
}

template <int DQK, int VB>
static int launch_att(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const AttParams& prm,
                      int n_tiles, cudaStream_t s) {
    using Cfg = AttCfg<DQK, VB>;
    auto kern = attention_tc_kernel<DQK, VB>;
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM) != cudaSuccess) return -3;
        attr = true;
    }
    const long grid = (long)n_tiles * prm.nkv * prm.nsplit;
    if (grid <= 0) return 0;
    kern<<<(unsigned)grid, ATT_THREADS, Cfg::SMEM, s>>>(tq, tk, tv, prm);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int attention_tc(const bf16_t* q, const bf16_t* k, const bf16_t* v, bf16_t* out, long rows, const AttnTile* tiles,
                 int n_tiles, int nh, int nkv, int hd, int window, cudaStream_t s) {
    if (rows <= 0 || n_tiles <= 0) return 0;
    if ((hd != 256 && hd != 512) || !attention_tc_tile_tokens(nh, nkv, hd)) return -1;
    const int G = nh / nkv;
    const int tq = 128 / G;  // query tokens per CTA (128 MMA rows)
    CUtensorMap mq, mk, mv;
    const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    // q [rows, nh, hd]: box (64 ch, G heads, tq tokens) -> 128 rows of 128 B.
    if (make_tmap_3d(&mq, dt, q, hd, nh, rows, (uint64_t)hd * 2, (uint64_t)nh * hd * 2, 64, G, tq) ||
        make_tmap_3d(&mk, dt, k, hd, nkv, rows, (uint64_t)hd * 2, (uint64_t)nkv * hd * 2, 64, 1, ATT_BN) ||
        make_tmap_3d(&mv, dt, v, hd, nkv, rows, (uint64_t)hd * 2, (uint64_t)nkv * hd * 2, 64, 1, hd == 256 ? AP_BN : ATT_BN))
        return -1;
    AttParams prm;
    prm.tiles = tiles;
    prm.out = out;
    prm.nh = nh;
    prm.nkv = nkv;
    prm.hd = hd;
    prm.window = window;
    prm.G = G;
    prm.tq = tq;
    prm.nsplit = hd / ATT_DV;
    if (hd == 256) {
        // CTA pairs: clusters of 2, one per (pair tile, K/V head).
        static bool attr = false;
        if (!attr) {
            if (cudaFuncSetAttribute(attention_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ApCfg::SMEM) !=
                cudaSuccess)
                return -3;
            attr = true;
        }
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute la[1];
        la[0].id = cudaLaunchAttributeClusterDimension;
        la[0].val.clusterDim.x = 2;
        la[0].val.clusterDim.y = 1;
        la[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3((unsigned)(2L * n_tiles * nkv), 1, 1);
        cfg.blockDim = dim3(AP_THREADS, 1, 1);
        cfg.dynamicSmemBytes = ApCfg::SMEM;
        cfg.stream = s;
        cfg.attrs = la;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, attention_pair_kernel, mq, mk, mv, prm) == cudaSuccess ? 0 : -3;
    }
    // V buffers: as many as shared memory holds next to Q and the K ring (224 KB).
    return launch_att<512, 2>(mq, mk, mv, prm, n_tiles, s);
}

}  // namespace eg2

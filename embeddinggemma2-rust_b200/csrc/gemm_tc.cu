// Projection GEMMs on the 5th-generation tensor cores: C[M, N] = A[M, K] . W[N, K]^T with both
// operands K-major (nn.Linear layout), fp32 accumulation in tensor memory.
//
// Replaces the reference's cuBLAS calls `Gpu::gemm_bf16` (src/gpu/mod.rs:600-630, cublasGemmEx
// bf16 -> f32 accumulate) and `Gpu::matmul_nt` in TF32 mode (src/gpu/mod.rs:554-577), plus the
// elementwise kernels that follow them: `gelu_mul_gu` (kernels.cu:239-246, fused as EPI_GELU_GU),
// `ple_gate` (kernels.cu:294-299, fused as EPI_PLE_GATE) and `qkv_post` (kernels.cu:183-237,
// fused as EPI_QKV for head widths that tile the 256 output columns).
//
// Structure (one CTA per SM, persistent over output tiles of 128 x BN):
//   warp 0       TMA producer: A tile [128 x 64 bf16] and W tile [BN x 64] per stage, 128 B swizzle
//   warp 1       TMEM allocation; lane 0 issues tcgen05.mma (M=128, N=BN, K=16) and commits
//   warps 2..9   two epilogue sets of 4 warps (one warp per TMEM lane quadrant). Set s owns TMEM
//                accumulator s and the CTA's tiles of parity s, so two tiles' epilogues run at once
//                while the MMAs of a third fill the free accumulator: the epilogues (norms, RoPE,
//                GELU) are latency-bound and need the extra warps to overlap the main loop.
//
// EPI_ADD_NORM and EPI_GROUP_NORM launch clusters of two CTAs: CTA rank r computes columns
// [256 r, 256 r + 256) of each 512-column group, and the per-row sums of squares of the two halves are
// swapped through distributed shared memory (st.async into the peer's slot, completing bytes on the
// peer's mbarrier).
#include "common.cuh"
#include "kernels.h"

namespace eg2 {

template <typename TIn>
struct InTraits;
template <>
struct InTraits<bf16_t> {
    static constexpr int BK = 64;  // elements per 128-byte row
    static constexpr uint32_t FMT = 1;
};
template <>
struct InTraits<float> {
    static constexpr int BK = 32;
    static constexpr uint32_t FMT = 2;  // tf32
};

constexpr int GEMM_BM = 128;
constexpr int GEMM_THREADS = 320;
// WIDE (the sliding-layer QKV epilogue): 16 epilogue warps, two per TMEM lane quadrant and set, each
// taking half of the tile's columns. That epilogue is latency-bound (~0.3 IPC per warp) and longer than
// the main loop, so with two accumulators the tile period is (epilogue + main loop) / 2.
constexpr int gemm_threads(bool wide) { return wide ? 576 : GEMM_THREADS; }

// PAIR: 2-CTA clusters computing 256 x BN tiles with tcgen05.mma.cta_group::2 (M = 256): each CTA
// loads its own 128 rows of A and half (BN / 2 rows) of B, so per SM a K block moves 32 KB into and
// 32 KB out of shared memory instead of 48 + 48 KB -- the single-CTA tile needs ~190 B/cycle of shared
// memory at the full tensor rate, more than shared memory delivers.
// TIO: the epilogue's global I/O goes through TMA, each epilogue warp owning four 2 KB
// shared-memory slots (instead of the 2.5 KB staging tile of the register path) -- EPI_ADD_NORM
// for its residual reads and h / t writes, EPI_PLE_GATE for its PLE inputs and outputs, EPI_QKV
// and EPI_GELU_GU for their outputs. The main loop gives up stages for them.
// DUAL (EPI_PLE_FUSED): two products per tile, each BN = 128 wide, in four TMEM accumulators (two per
// epilogue set); 32 KB stages, four of them.
// NP: CTAs per row group of the add-norm cluster epilogue (2: 512-wide rows, the text tower; 3: 768, the
// vision tower), each owning 256 columns; their row sums of squares go to every other CTA of the cluster.
template <int BN, bool PAIR = false, bool TIO = false, bool WIDE = false, bool DUAL = false, int NP = 2>
struct GemmCfg {
    static constexpr int NEPI = WIDE ? 16 : 8;  // epilogue warps
    static constexpr int A_BYTES = GEMM_BM * 128;
    static constexpr int B_BYTES = (PAIR ? BN / 2 : BN) * 128;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = DUAL ? 4 : TIO ? (PAIR ? 4 : 3) : PAIR ? 6 : (BN == 256) ? 4 : 6;
    // Barriers follow the stages; TIO slots must start on a 1 KB boundary.
    static constexpr int OFF_STAGE = STAGES * STAGE_BYTES + (TIO ? 1024 : 256);
    // 32 rows x 64 B + 16 B pad; TIO: four 2 KB slots (WIDE: two)
    static constexpr int STAGE_WARP = TIO ? (WIDE ? 4096 : 8192) : 32 * (64 + 16);
    static constexpr int OFF_W = OFF_STAGE + NEPI * STAGE_WARP;  // EPI_QKV: norm weights, inv freqs
    // EPI_QKV: norm weights + inverse frequencies (<= 3 KB). Cluster modes: this CTA's halves of the
    // norm weights (EPI_QKV_PAIR: wq, wk and 128 inverse frequencies, 2.5 KB), exchange slots
    // [set][slot][128 rows] at +X_OFF (2 KB), exchange barriers [set][slot] at +XB_OFF.
    // WIDE: the two half-warps' partial sums of squares [set][quadrant][slot][half][32] (4 KB) at
    // +XW_OFF, their barriers [set][quadrant][slot] at +XWB_OFF.
    // DUAL: exchange slots [set][slot][source rank 0..3][128 rows] (8 KB); NP = 3 the same with 3 sources.
    static constexpr int X_OFF = 2560;
    static constexpr int XB_OFF = X_OFF + ((DUAL || NP > 2) ? 8192 : 2048);
    static constexpr int XW_OFF = XB_OFF + 64;
    static constexpr int XWB_OFF = XW_OFF + 4096;
    static constexpr int W_BYTES = WIDE ? XWB_OFF + 128 : XB_OFF + 64;
    static constexpr int SMEM_BYTES = 1024 + OFF_W + W_BYTES;
    static constexpr uint32_t TMEM_COLS = DUAL ? 4 * BN : 2 * BN;
};

// GELU (tanh form) for the tensor-core epilogues: 0.5 x (1 + tanh(u)) = x * sigmoid(2 u), with
// sigmoid via ex2 and a fast reciprocal; within ~2e-7 relative of gelu_tanh_f (which the
// float32 path keeps), far below the bf16 / TF32 rounding these results go through.
EG2_DEV float gelu_fast(float x) {
    const float u = 0.79788456f * (x + 0.044715f * x * x * x);
    return __fdividef(x, 1.f + ex2_approx(-2.8853900817779268f * u));  // 2 log2(e) u
}

// Warp-cooperative store of a 32-row x 32-column chunk (lane i holds row row0 + i): each 64-byte
// row segment goes through the warp's padded shared-memory tile, then every store instruction
// writes whole 64-byte segments of 8 rows instead of 32 scattered 16-byte pieces. f32 chunks go
// in two 16-column halves. Rows >= M are skipped. All 32 lanes must call it.
template <typename TOut>
EG2_DEV void warp_store32(TOut* out, long ldo, int row0, int M, long col, const float (&v)[32], uint8_t* stage) {
    const int lane = threadIdx.x & 31;
    constexpr int STRIDE = 64 + 16;
    constexpr int COLS = 64 / (int)sizeof(TOut);  // columns per 64-byte segment
#pragma unroll
    for (int h = 0; h < 32 / COLS; h++) {
        uint8_t* my = stage + lane * STRIDE;
        if constexpr (sizeof(TOut) == 2) {
#pragma unroll
            for (int q = 0; q < 4; q++)
                *reinterpret_cast<uint4*>(my + q * 16) =
                    make_uint4(bf16x2_bits(v[8 * q + 0], v[8 * q + 1]), bf16x2_bits(v[8 * q + 2], v[8 * q + 3]),
                               bf16x2_bits(v[8 * q + 4], v[8 * q + 5]), bf16x2_bits(v[8 * q + 6], v[8 * q + 7]));
        } else {
#pragma unroll
            for (int q = 0; q < 4; q++)
                *reinterpret_cast<float4*>(my + q * 16) =
                    make_float4(v[16 * h + 4 * q], v[16 * h + 4 * q + 1], v[16 * h + 4 * q + 2], v[16 * h + 4 * q + 3]);
        }
        __syncwarp();
#pragma unroll
        for (int p = lane; p < 32 * 4; p += 32) {
            const int r = p >> 2, sg = p & 3;
            if (row0 + r < M)
                *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(out + (long)(row0 + r) * ldo + col + h * COLS) + sg * 16) =
                    *reinterpret_cast<const uint4*>(stage + r * STRIDE + sg * 16);
        }
        __syncwarp();
    }
}

// EPI_QKV: the tile's BN columns are whole heads of one kind (q, k or v). Pass 1 reads the
// accumulator for the per-head sums of squares; pass 2 reads it again, normalises (q / k times
// their norm weights), applies RoPE to q / k (split-halves rule, pairs i and i + part / 2) and
// stores the heads. Operation for operation the arithmetic of qkv_post_kernel (rowops.cu), except
// that the RoPE angle pos * inv_freq (computed in f32 like the reference's tables, src/ops.rs:303-306)
// goes through sincos_reduced instead of a table. All 32 lanes run every tcgen05.ld; rows past M
// only skip the stores.
// Tensor maps of the epilogue's TMA I/O (TIO). EPI_ADD_NORM: [0] residual h (f32, 16 x 32 boxes),
// [1] t (bf16, 32 x 32); EPI_QKV: [0..2] q, k, v; EPI_PLE_GATE: [0] the output (bf16, 32 x 32). All
// with the 64-byte swizzle.
struct alignas(64) EpiMaps {
    CUtensorMap m[3];
};

// TIO store of a 32-row x 32-column bf16 chunk (lane i holds row i) at (x, y) of map m, through
// slot n % NSLOT of the warp's 2 KB slots (64-byte swizzle: row r's 16-byte unit j at
// r * 64 + 16 * (j ^ ((r >> 1) & 3)), conflict-free for lane = row). The slot's previous store (the
// NSLOT-th newest bulk group of lane 0) must have been read out first. Rows past the tensor are not
// written. All 32 lanes call it with the same n.
template <int NSLOT = 4>
EG2_DEV void tio_store32(const CUtensorMap* m, uint8_t* slots, int n, const float (&v)[32], int x, int y) {
    const int lane = threadIdx.x & 31;
    uint8_t* buf = slots + (n % NSLOT) * 2048;
    if (lane == 0) bulk_wait_read<NSLOT - 1>();
    __syncwarp();
    const uint32_t sw = (uint32_t)((lane >> 1) & 3);
    uint8_t* row = buf + lane * 64;
#pragma unroll
    for (int j = 0; j < 4; j++)
        *reinterpret_cast<uint4*>(row + ((j ^ sw) << 4)) =
            make_uint4(bf16x2_bits(v[8 * j], v[8 * j + 1]), bf16x2_bits(v[8 * j + 2], v[8 * j + 3]),
                       bf16x2_bits(v[8 * j + 4], v[8 * j + 5]), bf16x2_bits(v[8 * j + 6], v[8 * j + 7]));
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(m, buf, x, y);
        bulk_commit();
    }
}

// EPI_QKV, 256-wide heads, WIDE: this warp takes half hw of the tile's 128 rotation pairs (pairs
// 64 hw .. 64 hw + 63: columns 64 hw.. and 128 + 64 hw..), in sub-chunks of 16 pairs. The head's sum of
// squares is completed with the other half's partial (the other warp of this TMEM lane quadrant and
// set): both write their partial to slot X % 2 and meet on that slot's mbarrier (64 arrivals, bounded
// wait); a slot is rewritten only after the partner has passed the next meeting, i.e. has read it.
// Outputs (16 columns of bf16 per store, 32-byte swizzle: row r's 16-byte unit j at
// r * 32 + 16 * (j ^ ((r >> 2) & 1))) leave by TMA store through the warp's two 2 KB slots, a
// sub-chunk's x1 and x2 pieces sharing a slot, a proxy fence and a bulk group. Same arithmetic as
// epilogue_qkv256 except the order in which the sum of squares is added up. Returns false when a wait
// ran out.
EG2_DEV bool epilogue_qkv256_wide(const QkvEpilogue& Q, uint32_t tbase, int row0, int M, int n0, uint8_t* slots,
                                  const float* wsm, const EpiMaps& em, int& nst, int hw, float* xv, uint64_t* xb,
                                  int& X, volatile int* abort_flag) {
    const int lane = threadIdx.x & 31;
    const int row = row0 + lane;
    const int qw = Q.nh * 256, kw = Q.nkv * 256;
    int head, which;
    const float* w;
    bool rot;
    if (n0 < qw) {
        head = n0 >> 8, w = wsm, rot = true, which = 0;
    } else if (n0 < qw + kw) {
        head = (n0 - qw) >> 8, w = wsm + 256, rot = true, which = 1;
    } else {
        head = (n0 - qw - kw) >> 8, w = nullptr, rot = false, which = 2;
    }
    const bool live = row < M;
    const float pf = (rot && live) ? (float)(Q.pos ? Q.pos[(long)row * Q.pos_stride] : row) : 0.f;
    const int c0 = 64 * hw;  // this half's first pair
    float ss = 0.f;
#pragma unroll 1
    for (int c = 0; c < 64; c += 32) {
        uint32_t r0[32], r1[32];
        tmem_ld32(tbase + c0 + c, r0);
        tmem_ld32(tbase + 128 + c0 + c, r1);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; j++) {
            ss = fmaf(__uint_as_float(r0[j]), __uint_as_float(r0[j]), ss);
            ss = fmaf(__uint_as_float(r1[j]), __uint_as_float(r1[j]), ss);
        }
    }
    {
        float* slot = xv + (X & 1) * 64;
        slot[hw * 32 + lane] = ss;
        mbar_arrive(&xb[X & 1]);
        if (!mbar_wait(&xb[X & 1], (X >> 1) & 1, EG2_DEV_TIMEOUT_GEMM, abort_flag)) return false;
        ss += *reinterpret_cast<volatile float*>(slot + (hw ^ 1) * 32 + lane);
        X++;
    }
    const float inv = 1.0f / sqrtf(ss / 256.f + Q.eps);
    const float* invs = wsm + 512;
    const int col1 = head * 256;
    const uint32_t sw32 = (uint32_t)((lane >> 2) & 1);
    // A sub-chunk's two 16-column pieces (x1 at col, x2 at col + 128) go into the two 1 KB halves of
    // slot nst % 2 behind one proxy fence, then lane 0 issues both TMA stores as one bulk group.
    auto store_pair = [&](const float (&v1)[16], const float (&v2)[16], int col) {
        uint32_t p1[8], p2[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            p1[j] = bf16x2_bits(v1[2 * j], v1[2 * j + 1]);
            p2[j] = bf16x2_bits(v2[2 * j], v2[2 * j + 1]);
        }
        uint8_t* buf = slots + (nst & 1) * 2048;
        if (lane == 0) bulk_wait_read<1>();  // the slot's previous stores are read out
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 2; j++) {
            *reinterpret_cast<uint4*>(buf + lane * 32 + ((j ^ sw32) << 4)) =
                make_uint4(p1[4 * j], p1[4 * j + 1], p1[4 * j + 2], p1[4 * j + 3]);
            *reinterpret_cast<uint4*>(buf + 1024 + lane * 32 + ((j ^ sw32) << 4)) =
                make_uint4(p2[4 * j], p2[4 * j + 1], p2[4 * j + 2], p2[4 * j + 3]);
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
            tma_store_2d(&em.m[which], buf, col, row0);
            tma_store_2d(&em.m[which], buf + 1024, col + 128, row0);
            bulk_commit();
        }
        nst++;
    };
#pragma unroll 1
    for (int sc = 0; sc < 4; sc++) {
        const int p = c0 + 16 * sc;  // first pair of the sub-chunk
        float x1[16], x2[16];
        {
            uint32_t a[16], b[16];
            tmem_ld16(tbase + p, a);
            tmem_ld16(tbase + 128 + p, b);
            tmem_ld_wait();
#pragma unroll
            for (int t = 0; t < 16; t++) {
                x1[t] = __uint_as_float(a[t]) * inv;
                x2[t] = __uint_as_float(b[t]) * inv;
            }
        }
        if (rot) {
#pragma unroll
            for (int t = 0; t < 16; t++) {
                const float a1 = x1[t] * w[p + t], a2 = x2[t] * w[128 + p + t];
                float sj, cj;
                sincos_reduced(pf * invs[p + t], sj, cj);
                x1[t] = a1 * cj - a2 * sj;
                x2[t] = a2 * cj + a1 * sj;
            }
        }
        store_pair(x1, x2, col1 + p);
    }
    return true;
}

// EPI_QKV with one 256-wide head per tile and RoPE over the whole head (pairs i, i + 128): the same
// arithmetic as the general form below with the head geometry known at compile time, the position
// read once per tile (before pass 1, so its latency hides behind the TMEM reads) and two TMEM loads
// in flight per wait.
template <typename TOut>
EG2_DEV void epilogue_qkv256(const QkvEpilogue& Q, uint32_t tbase, int row0, int M, int n0, uint8_t* stage,
                             const float* wsm) {
    const int row = row0 + (int)(threadIdx.x & 31);
    const int qw = Q.nh * 256, kw = Q.nkv * 256;
    TOut* base;
    int nheads, head;
    const float* w;
    bool rot;
    int which;
    if (n0 < qw) {
        base = (TOut*)Q.q, nheads = Q.nh, head = n0 >> 8, w = wsm, rot = true, which = 0;
    } else if (n0 < qw + kw) {
        base = (TOut*)Q.k, nheads = Q.nkv, head = (n0 - qw) >> 8, w = wsm + 256, rot = true, which = 1;
    } else {
        base = (TOut*)Q.v, nheads = Q.nkv, head = (n0 - qw - kw) >> 8, w = nullptr, rot = false, which = 2;
    }
    const bool live = row < M;
    const float pf = (rot && live) ? (float)(Q.pos ? Q.pos[(long)row * Q.pos_stride] : row) : 0.f;
    float ss = 0.f;
#pragma unroll 1
    for (int c = 0; c < 8; c += 2) {
        uint32_t r0[32], r1[32];
        tmem_ld32(tbase + c * 32, r0);
        tmem_ld32(tbase + c * 32 + 32, r1);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; j++) {
            ss = fmaf(__uint_as_float(r0[j]), __uint_as_float(r0[j]), ss);
            ss = fmaf(__uint_as_float(r1[j]), __uint_as_float(r1[j]), ss);
        }
    }
    const float inv = 1.0f / sqrtf(ss / 256.f + Q.eps);
    const float* invs = wsm + 512;
    const long ldo = (long)nheads * 256, col1 = (long)head * 256;
#pragma unroll 1
    for (int c = 0; c < 4; c++) {
        float x1[32], x2[32];
        {
            uint32_t a[32], b[32];
            tmem_ld32(tbase + c * 32, a);
            tmem_ld32(tbase + 128 + c * 32, b);
            tmem_ld_wait();
#pragma unroll
            for (int t = 0; t < 32; t++) {
                x1[t] = __uint_as_float(a[t]) * inv;
                x2[t] = __uint_as_float(b[t]) * inv;
            }
        }
        if (rot) {
#pragma unroll
            for (int t = 0; t < 32; t++) {
                const float a1 = x1[t] * w[c * 32 + t], a2 = x2[t] * w[128 + c * 32 + t];
                float sj, cj;
                sincos_reduced(pf * invs[c * 32 + t], sj, cj);
                x1[t] = a1 * cj - a2 * sj;
                x2[t] = a2 * cj + a1 * sj;
            }
        }
        warp_store32<TOut>(base, ldo, row0, M, col1 + c * 32, x1, stage);
        warp_store32<TOut>(base, ldo, row0, M, col1 + 128 + c * 32, x2, stage);
    }
}

template <typename TOut, int BN>
EG2_DEV void epilogue_qkv(const GemmEpilogue& epi, uint32_t tbase, int row0, int M, int n0, uint8_t* stage,
                          const float* wsm) {
    const int row = row0 + (int)(threadIdx.x & 31);
    const QkvEpilogue& Q = epi.qkv;
    if constexpr (BN == 256) {
        if (Q.hd == 256 && Q.part == 256) {
            epilogue_qkv256<TOut>(Q, tbase, row0, M, n0, stage, wsm);
            return;
        }
    }
    const int hd = Q.hd, qw = Q.nh * hd, kw = Q.nkv * hd;
    TOut* base;
    int nheads, head0;
    const float* w;
    bool rot;
    if (n0 < qw) {
        base = (TOut*)Q.q, nheads = Q.nh, head0 = n0 / hd, w = wsm, rot = true;
    } else if (n0 < qw + kw) {
        base = (TOut*)Q.k, nheads = Q.nkv, head0 = (n0 - qw) / hd, w = wsm + hd, rot = true;
    } else {
        base = (TOut*)Q.v, nheads = Q.nkv, head0 = (n0 - qw - kw) / hd, w = nullptr, rot = false;
    }
    float ss[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
    for (int c = 0; c < BN / 32; c++) {
        uint32_t r[32];
        tmem_ld32(tbase + c * 32, r);
        tmem_ld_wait();
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < 32; j++) s = fmaf(__uint_as_float(r[j]), __uint_as_float(r[j]), s);
        const int hi = (c * 32) / hd;
#pragma unroll
        for (int q = 0; q < 4; q++)
            if (q == hi) ss[q] += s;
    }
    float inv[4];
#pragma unroll
    for (int q = 0; q < 4; q++) inv[q] = 1.0f / sqrtf(ss[q] / (float)hd + Q.eps);
    const bool live = row < M;
    const int half = Q.part / 2;
    const float* invs = wsm + 2 * hd;
    const long ldo = (long)nheads * hd;
#pragma unroll 1
    for (int c = 0; c < BN / 32; c++) {
        const int col0 = c * 32, hi = col0 / hd, hc = col0 % hd;
        float iv = inv[0];
#pragma unroll
        for (int q = 1; q < 4; q++)
            if (q == hi) iv = inv[q];
        const long col_base = (long)(head0 + hi) * hd;
        if (!rot) {
            uint32_t r[32];
            tmem_ld32(tbase + col0, r);
            tmem_ld_wait();
            float o[32];
#pragma unroll
            for (int t = 0; t < 32; t++) o[t] = __uint_as_float(r[t]) * iv;
            warp_store32<TOut>(base, ldo, row0, M, col_base + hc, o, stage);
        } else if (half >= 32) {
            if ((hc % Q.part) >= half) continue;  // written together with its partner chunk
            const int pi = hc / Q.part, j0 = hc % Q.part;
            const float pf = live ? (float)(Q.pos ? Q.pos[(long)row * Q.pos_stride + pi] : row) : 0.f;
            float x1[32], x2[32];
            {
                uint32_t a[32], b[32];
                tmem_ld32(tbase + col0, a);
                tmem_ld32(tbase + col0 + half, b);
                tmem_ld_wait();
#pragma unroll
                for (int t = 0; t < 32; t++) {
                    x1[t] = __uint_as_float(a[t]) * iv * w[hc + t];
                    x2[t] = __uint_as_float(b[t]) * iv * w[hc + half + t];
                }
            }
#pragma unroll
            for (int t = 0; t < 32; t++) {
                float sj, cj;
                sincos_reduced(pf * invs[j0 + t], sj, cj);
                const float a1 = x1[t], a2 = x2[t];
                x1[t] = a1 * cj - a2 * sj;
                x2[t] = a2 * cj + a1 * sj;
            }
            warp_store32<TOut>(base, ldo, row0, M, col_base + hc, x1, stage);
            warp_store32<TOut>(base, ldo, row0, M, col_base + hc + half, x2, stage);
        } else {
            // part == 32: both halves of each rotated pair lie in this chunk.
            const int pi = hc / Q.part;
            const float pf = live ? (float)(Q.pos ? Q.pos[(long)row * Q.pos_stride + pi] : row) : 0.f;
            float o[32];
            {
                uint32_t a[32];
                tmem_ld32(tbase + col0, a);
                tmem_ld_wait();
#pragma unroll
                for (int t = 0; t < 32; t++) o[t] = __uint_as_float(a[t]) * iv * w[hc + t];
            }
#pragma unroll
            for (int t = 0; t < 16; t++) {
                float sj, cj;
                sincos_reduced(pf * invs[t], sj, cj);
                const float a1 = o[t], a2 = o[t + 16];
                o[t] = a1 * cj - a2 * sj;
                o[t + 16] = a2 * cj + a1 * sj;
            }
            warp_store32<TOut>(base, ldo, row0, M, col_base + hc, o, stage);
        }
    }
}

// Lane i loads the 16-byte segments p = i + 32 q (q = 0..7) of a 32-row x 32-column f32 chunk:
// row p / 8, columns 4 (p % 8) .. + 3; every load instruction covers four whole 128-byte row
// segments. Rows >= M read as zeros. warp_load32_finish hands lane i the 32 values of row i
// through the warp's staging tile (two 16-column halves, as warp_store32).
EG2_DEV void warp_load32_issue(const float* src, long ld, int row0, int M, long col, uint4 (&b)[8]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int q = 0; q < 8; q++) {
        const int r = (lane >> 3) + 4 * q;
        b[q] = (row0 + r < M) ? *(reinterpret_cast<const uint4*>(src + (long)(row0 + r) * ld + col) + (lane & 7))
                              : make_uint4(0u, 0u, 0u, 0u);
    }
}
EG2_DEV void warp_load32_finish(const uint4 (&b)[8], float (&v)[32], uint8_t* stage) {
    const int lane = threadIdx.x & 31;
    constexpr int STRIDE = 64 + 16;
    const int sg = lane & 7;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        if ((sg >> 2) == h) {
#pragma unroll
            for (int q = 0; q < 8; q++)
                *reinterpret_cast<uint4*>(stage + ((lane >> 3) + 4 * q) * STRIDE + (sg & 3) * 16) = b[q];
        }
        __syncwarp();
#pragma unroll
        for (int s4 = 0; s4 < 4; s4++) {
            const float4 x = *reinterpret_cast<const float4*>(stage + lane * STRIDE + s4 * 16);
            v[16 * h + 4 * s4 + 0] = x.x;
            v[16 * h + 4 * s4 + 1] = x.y;
            v[16 * h + 4 * s4 + 2] = x.z;
            v[16 * h + 4 * s4 + 3] = x.w;
        }
        __syncwarp();
    }
}

// em: the tensor maps of the epilogue's TMA I/O (TIO only).
template <typename TIn, int BN, int EPI, typename TOut, bool PAIR = false, bool TIO = false, bool WIDE = false, int NP = 2>
__global__ void __launch_bounds__(gemm_threads(WIDE), 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ EpiMaps em, int M, int N, int K, GemmEpilogue epi) {
    static_assert(!WIDE || (EPI == EPI_QKV && PAIR && TIO) || (EPI == EPI_QKV_PAIR && TIO),
                  "WIDE: the QKV epilogues with TMA stores");
    constexpr int NTHREADS = gemm_threads(WIDE);
    static_assert(!TIO || (BN == 256 && (EPI == EPI_ADD_NORM || EPI == EPI_GROUP_NORM || EPI == EPI_QKV_PAIR ||
                                         (PAIR && (EPI == EPI_QKV || EPI == EPI_PLE_GATE || EPI == EPI_GELU_GU)))) ||
                      (BN == 128 && EPI == EPI_PLE_FUSED && !PAIR),
                  "TMA epilogue I/O: the cluster epilogues, and the pair QKV / PLE-gate / GELU epilogues");
    constexpr bool DUAL = EPI == EPI_PLE_FUSED;
    static_assert(NP == 2 || (NP == 3 && EPI == EPI_ADD_NORM && !PAIR), "NP = 3: the single-CTA add-norm epilogue");
    using Cfg = GemmCfg<BN, PAIR, TIO, WIDE, DUAL, NP>;
    constexpr int BK = InTraits<TIn>::BK;
    constexpr int STAGES = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;  // PAIR: the MMA issuer's final wait for its own MMAs
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint64_t* hbar = drain + 2;  // TIO: [epilogue warp][slot] residual-load barriers

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_m = (M + GEMM_BM - 1) / GEMM_BM, tiles_n = N / BN;
    const int kblocks = K / BK;
    // This CTA's tiles: linear ids t_first + i * t_step < t_count. Cluster modes: the cluster's
    // (row block, 512-column group) pairs, the 256-column half fixed by the CTA's rank.
    // PAIR: the cluster's 256-row x BN tiles, this CTA's 128 rows fixed by its rank.
    constexpr bool AN = EPI == EPI_ADD_NORM;
    constexpr bool CL = AN || EPI == EPI_GROUP_NORM || EPI == EPI_QKV_PAIR || DUAL;
    // QUAD: a cluster epilogue on CTA-pair MMAs -- clusters of four CTAs, two MMA pairs. Cluster rank
    // r: MMA pair r >> 1 computes columns [256 (r >> 1), +256) of each 512-column group, its CTA r & 1
    // rows [128 (r & 1), +128) of the cluster's 256-row block; the row sums of squares are exchanged
    // with rank r ^ 2, which holds the same rows' other column half.
    constexpr bool QUAD = CL && PAIR;
    static_assert(!QUAD || EPI == EPI_ADD_NORM || EPI == EPI_GROUP_NORM, "QUAD: the add-norm and group-norm epilogues");
    static_assert(!PAIR || sizeof(TIn) == 2, "CTA-pair MMAs are bf16 only");
    const int GW = DUAL ? 512 : 256 * NP;  // cluster modes: columns of one row group
    const int groups = N / GW;
    const uint32_t crank = (CL || PAIR) ? cluster_ctarank() : 0u;
    const uint32_t prow = PAIR ? (crank & 1u) : crank;       // PAIR: this CTA's row half of the pair tile
    const uint32_t pcol = QUAD ? (crank >> 1) : crank;       // cluster epilogues: column half of the group
    const uint32_t pair_base = crank & ~1u;                  // PAIR: the even CTA of this CTA's MMA pair
    const uint32_t xpeer = QUAD ? (crank ^ 2u) : (crank ^ 1u);  // CL: the CTA with the other column half
    const bool lead = PAIR ? prow == 0 : crank == 0;
    const int tiles_mp = (tiles_m + 1) / 2;
    constexpr int CSZ = (QUAD || DUAL) ? 4 : NP;  // cluster size
    const int t_first = (CL || PAIR) ? (int)(blockIdx.x / CSZ) : (int)blockIdx.x;
    const int t_step = (CL || PAIR) ? (int)(gridDim.x / CSZ) : (int)gridDim.x;
    // K split (EPI_STORE): linear id t = base tile * S + slice; slice s covers K blocks
    // [s * kbs, s * kbs + kbs).
    const int S = (EPI == EPI_STORE && epi.ksplit > 1) ? epi.ksplit : 1;
    // DUAL: K blocks [0, kblocks) feed the first product, [kblocks, 2 kblocks) the second.
    const int kbs = DUAL ? 2 * kblocks : kblocks / S;
    const int t_count = (QUAD ? tiles_mp * groups : CL ? tiles_m * groups : PAIR ? tiles_mp * tiles_n : tiles_m * tiles_n) * S;
    auto tile_m0 = [&](int t) {
        t /= S;
        if (QUAD) return (t / groups) * 2 * GEMM_BM + (int)prow * GEMM_BM;
        return PAIR ? (t / tiles_n) * 2 * GEMM_BM + (int)prow * GEMM_BM : (CL ? t / groups : t / tiles_n) * GEMM_BM;
    };
    auto tile_n0 = [&](int t) {
        t /= S;
        return CL ? (t % groups) * GW + (int)pcol * BN : (t % tiles_n) * BN;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(&tfull[a], 1);
            // Every epilogue thread of the set (PAIR: of both CTAs) frees the accumulator.
            mbar_init(&tempty[a], (WIDE ? 256 : 128) * (PAIR ? 2 : 1));
        }
        mbar_init(drain, 1);
        if constexpr (TIO && !WIDE) {
            for (int x = 0; x < 32; x++) mbar_init(&hbar[x], 1);
        }
        if constexpr (WIDE) {
            uint64_t* xb = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_W + Cfg::XWB_OFF);
            for (int x = 0; x < 16; x++) mbar_init(&xb[x], 64);  // both half-warps of a quadrant
        }
        if constexpr (CL) {
            uint64_t* xb = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_W + Cfg::XB_OFF);
            for (int x = 0; x < 4; x++) mbar_init(&xb[x], 1);  // one local arrival (expect_tx) per exchange
        }
        *abort_flag = 0;
        fence_mbarrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if constexpr (TIO) {  // the maps this epilogue uses
            tma_prefetch_desc(&em.m[0]);
            if constexpr (EPI != EPI_GELU_GU && EPI != EPI_GROUP_NORM) tma_prefetch_desc(&em.m[1]);
            if constexpr (EPI == EPI_QKV || EPI == EPI_QKV_PAIR || DUAL) tma_prefetch_desc(&em.m[2]);
        }
    }
    if constexpr (EPI == EPI_QKV) {
        // q_norm / k_norm weights and the inverse frequencies, once per CTA.
        float* wsm = reinterpret_cast<float*>(smem + Cfg::OFF_W);
        const int hd = epi.qkv.hd, nf = epi.qkv.part / 2;
        for (int i = threadIdx.x; i < 2 * hd + nf; i += NTHREADS)
            wsm[i] = i < hd ? epi.qkv.wq[i] : i < 2 * hd ? epi.qkv.wk[i - hd] : epi.qkv.inv_freq[i - 2 * hd];
    }
    if constexpr (EPI == EPI_QKV_PAIR) {
        // q_norm / k_norm weights for this CTA's 256 head channels (tile column t holds channel
        // 128 r + t, or 256 + 128 r + t - 128), then the inverse frequencies of its 128 rotated pairs.
        float* wsm = reinterpret_cast<float*>(smem + Cfg::OFF_W);
        const int r = (int)crank;
        for (int i = threadIdx.x; i < 2 * BN + 128; i += NTHREADS) {
            const int t = i & (BN - 1);
            const int ch = t < 128 ? 128 * r + t : 256 + 128 * r + (t - 128);
            wsm[i] = i < BN ? epi.qkv.wq[ch] : i < 2 * BN ? epi.qkv.wk[ch] : epi.qkv.inv_freq[128 * r + (i - 2 * BN)];
        }
    } else if constexpr (CL) {
        // This CTA's halves of the norm weights (the same for every 512-column group).
        float* wsm = reinterpret_cast<float*>(smem + Cfg::OFF_W);
        const int n0 = (int)pcol * BN;
        for (int i = threadIdx.x; i < 2 * BN; i += NTHREADS)
            wsm[i] = i < BN ? epi.an.w1[n0 + i] : (epi.an.w2 ? epi.an.w2[n0 + i - BN] : 0.f);
    }
    if (warp == 1) {
        if constexpr (PAIR)
            tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
        else
            tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // The peer CTA's barriers must be initialised before anyone arrives on them.
    if constexpr (CL || PAIR) cluster_sync();
    // Launched as a programmatic dependent: the prologue above ran while the previous kernel was
    // finishing; the next kernel may start its own now, and this one reads its inputs only once the
    // previous kernel has completed. With at most two tiles per CTA (passes of few rows, where the
    // kernel's start-up latency is a large part of its time) the producer waits later, after
    // requesting its first weight tiles (the weights do not depend on the previous kernel); warp 0's
    // other lanes touch no memory. Long passes keep the plain order: there a CTA's start-up is a small
    // part of its time.
    const bool early_w = t_count <= 2 * t_step;
    grid_dep_launch();
    if (warp != 0 || !early_w) grid_dep_wait();

    if (warp == 0) {
        if (lane == 0) {
            // Stage st's byte count, and its activation (A) and weight (B) tiles. A is requested first:
            // it comes from HBM, the weights mostly from L2.
            auto expect = [&](int st) {
                if constexpr (PAIR) {
                    // Both CTAs' bytes complete on the even CTA's barrier.
                    if (lead) mbar_arrive_expect_tx(&full[st], 2 * Cfg::STAGE_BYTES);
                } else {
                    mbar_arrive_expect_tx(&full[st], Cfg::STAGE_BYTES);
                }
            };
            auto load_a = [&](int st, int m0, int kb) {
                uint8_t* sa = smem + st * Cfg::STAGE_BYTES;
                if constexpr (PAIR)
                    tma_load_2d_pair(sa, &tmA, mapa_shared(smem_u32(&full[st]), pair_base), kb * BK, m0);
                else if (DUAL && kb >= kblocks)
                    tma_load_2d(sa, &em.m[1], &full[st], (kb - kblocks) * BK, m0);
                else
                    tma_load_2d(sa, &tmA, &full[st], kb * BK, m0);
            };
            auto load_b = [&](int st, int n0, int kb) {
                uint8_t* sa = smem + st * Cfg::STAGE_BYTES;
                if constexpr (PAIR)
                    tma_load_2d_pair(sa + Cfg::A_BYTES, &tmB, mapa_shared(smem_u32(&full[st]), pair_base), kb * BK,
                                     n0 + (int)prow * (BN / 2));
                else if (DUAL && kb >= kblocks)
                    tma_load_2d(sa + Cfg::A_BYTES, &em.m[2], &full[st], (kb - kblocks) * BK, epi.aux_off + n0);
                else
                    tma_load_2d(sa + Cfg::A_BYTES, &tmB, &full[st], kb * BK, n0);
            };
            // early_w: the first STAGES weight tiles go out before the wait for the previous kernel.
            int n_pre = 0;
            if (early_w) {
                for (int tile = t_first; tile < t_count && n_pre < STAGES; tile += t_step) {
                    const int kb0 = (tile % S) * kbs, n0 = tile_n0(tile);
                    for (int kb = kb0; kb < kb0 + kbs && n_pre < STAGES; kb++, n_pre++) {
                        expect(n_pre);
                        load_b(n_pre, n0, kb);
                    }
                }
                grid_dep_wait();
            }
            int stage = 0, e = 0;
            uint32_t phase = 0;
            for (int tile = t_first; tile < t_count; tile += t_step) {
                // (No L2 prefetch of the epilogue's inputs here: 128 bulk prefetches per tile from this
                // thread delayed the main loop's loads more than they saved -- measured on B200.)
                const int m0 = tile_m0(tile), n0 = tile_n0(tile);
                const int kb0 = (tile % S) * kbs;
                for (int kb = kb0; kb < kb0 + kbs; kb++, e++) {
                    if (e >= n_pre) {
                        if (!mbar_wait(&empty[stage], phase ^ 1, EG2_DEV_TIMEOUT_GEMM, abort_flag)) goto done;
                        expect(stage);
                        load_a(stage, m0, kb);
                        load_b(stage, n0, kb);
                    } else {
                        load_a(stage, m0, kb);
                    }
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && PAIR && lead) {
            // CTA-pair MMAs: M = 256 (A rows 0..127 here, 128..255 in the peer), B halves in both CTAs.
            constexpr uint32_t idesc = umma_idesc(2 * GEMM_BM, BN, InTraits<TIn>::FMT);
            const uint64_t da0 = umma_desc_sw128(smem_u32(smem), 16, 1024);
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            for (int tile = t_first; tile < t_count; tile += t_step, local++) {
                const int acc = local & 1;
                const uint32_t acc_phase = (local >> 1) & 1;
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1, EG2_DEV_TIMEOUT_GEMM, abort_flag)) goto done;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0; kb < kbs; kb++) {
                    if (!mbar_wait(&full[stage], phase, EG2_DEV_TIMEOUT_GEMM, abort_flag)) goto done;
                    tc_fence_after();
                    const uint64_t ad = da0 + (uint64_t)(stage * (Cfg::STAGE_BYTES >> 4));
                    const uint64_t bd = ad + (uint64_t)(Cfg::A_BYTES >> 4);
                    mma_bf16_pair(d_tmem, ad, bd, idesc, kb != 0);
#pragma unroll
                    for (int kk = 1; kk < 4; kk++) mma_bf16_pair(d_tmem, ad + 2 * kk, bd + 2 * kk, idesc, 1);
                    mma_commit_pair_both(&empty[stage], pair_base);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                mma_commit_pair_both(&tfull[acc], pair_base);
            }
        } else if (lane == 0 && !PAIR) {
            constexpr uint32_t idesc = umma_idesc(GEMM_BM, BN, InTraits<TIn>::FMT);
            // Descriptors are built once; a K step of 32 bytes adds 2 to the start-address field.
            const uint64_t da0 = umma_desc_sw128(smem_u32(smem), 16, 1024);
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            for (int tile = t_first; tile < t_count; tile += t_step, local++) {
                const int acc = local & 1;
                const uint32_t acc_phase = (local >> 1) & 1;
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1, EG2_DEV_TIMEOUT_GEMM, abort_flag)) goto done;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * (DUAL ? 2 * BN : BN);
                for (int kb = 0; kb < kbs; kb++) {
                    if (!mbar_wait(&full[stage], phase, EG2_DEV_TIMEOUT_GEMM, abort_flag)) goto done;
                    tc_fence_after();
                    const uint64_t ad = da0 + (uint64_t)(stage * (Cfg::STAGE_BYTES >> 4));
                    const uint64_t bd = ad + (uint64_t)(Cfg::A_BYTES >> 4);
                    // DUAL: the second product accumulates into the next BN columns.
                    const bool second = DUAL && kb >= kblocks;
                    const uint32_t d_acc = d_tmem + (second ? BN : 0);
                    const uint32_t first_k = (kb != 0 && kb != (DUAL ? kblocks : -1)) ? 1u : 0u;
                    mma_bf16_or_tf32<TIn>(d_acc, ad, bd, idesc, first_k);
#pragma unroll
                    for (int kk = 1; kk < 4; kk++) mma_bf16_or_tf32<TIn>(d_acc, ad + 2 * kk, bd + 2 * kk, idesc, 1);
                    mma_commit(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                mma_commit(&tfull[acc]);
            }
        }
    } else {
        const int e = warp & 3;           // TMEM lane quadrant this warp may access
        const int set = WIDE ? (warp - 2) >> 3 : (warp - 2) >> 2;  // epilogue set = accumulator it owns
        const int hw = WIDE ? ((warp - 2) >> 2) & 1 : 0;              // WIDE: half of the tile's columns
        const float* wsm = reinterpret_cast<const float*>(smem + Cfg::OFF_W);
        uint8_t* stage = smem + Cfg::OFF_STAGE + (warp - 2) * Cfg::STAGE_WARP;
        TOut* out = reinterpret_cast<TOut*>(epi.out);
        // TIO: residual chunk g (16 columns; 16 per tile) goes to slot g % 4 of this warp, its load
        // completing phase (g / 4) % 2 of hb[g % 4]. Loads issued / chunks consumed so far:
        uint64_t* hb = hbar + (WIDE ? 0 : (warp - 2) * 4);
        int xq = 0;  // WIDE: sum-of-squares meetings so far
        int ld_issued = 0, ld_used = 0;
        int nst = 0;  // TIO output stores issued by this warp (slot nst % 4)
        int k = 0;    // tiles this set has taken: its k-th completion of tfull[set]
        for (int tile = t_first + set * t_step; tile < t_count; tile += 2 * t_step, k++) {
            if constexpr (TIO && (EPI == EPI_ADD_NORM || EPI == EPI_PLE_GATE)) {
                // Chunks 0-2 of this tile's residual (PLE inputs), before the accumulator is ready;
                // the slots' last TMA stores (the previous tile's outputs) must have been read out.
                if (lane == 0) {
                    bulk_wait_read<0>();
                    const int hr = tile_m0(tile) + 32 * e, hc = tile_n0(tile);
                    for (int c = 0; c < 3; c++) {
                        mbar_arrive_expect_tx(&hb[c], 2048);
                        tma_load_2d(stage + c * 2048, &em.m[EPI == EPI_ADD_NORM ? 0 : 1], &hb[c], hc + 16 * c, hr);
                    }
                }
                ld_issued += 3;
            }
            if (!mbar_wait(&tfull[set], k & 1, EG2_DEV_TIMEOUT_GEMM, abort_flag)) break;
            tc_fence_after();
            const int m0 = tile_m0(tile), n0 = tile_n0(tile);
            const int row0 = m0 + 32 * e, row = row0 + lane;
            const uint32_t tbase = tmem_base + ((uint32_t)(32 * e) << 16) + set * (DUAL ? 2 * BN : BN);
            // Cluster modes: sends this row's partial sum to the peer CTA (same slot there, st.async
            // counting 4 bytes on the peer's barrier) and returns the total once the peer's 128 values
            // (512 bytes, expected by this set's first thread) have landed here. Both CTAs add the same
            // two numbers, so both use the same norm.
            bool ok = true;
            auto exchange = [&](float part, int slot, uint32_t parity) -> float {
                float* xv = reinterpret_cast<float*>(smem + Cfg::OFF_W + Cfg::X_OFF);  // [set][slot][128]
                uint64_t* xb = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_W + Cfg::XB_OFF);
                const int rl = 32 * e + lane;
                if constexpr (NP > 2) {
                    // Every other CTA of the cluster gets this partial in its slot [set][slot][this rank];
                    // all add the NP partials in rank order, so every CTA uses the same norm.
                    const int x = set * 2 + slot;
                    float* slots = xv + x * NP * 128;
                    if (rl == 0) mbar_arrive_expect_tx(&xb[x], (NP - 1) * 128 * 4);
#pragma unroll
                    for (uint32_t pr = 0; pr < (uint32_t)NP; pr++)
                        if (pr != crank)
                            st_async_f32(mapa_shared(smem_u32(slots + crank * 128 + rl), pr), part,
                                         mapa_shared(smem_u32(&xb[x]), pr));
                    if (!mbar_wait(&xb[x], parity, EG2_DEV_TIMEOUT_GEMM, abort_flag)) {
                        ok = false;
                        return 0.f;
                    }
                    float tot = 0.f;
#pragma unroll
                    for (int src = 0; src < NP; src++)
                        tot += (src == (int)crank) ? part : *reinterpret_cast<volatile float*>(slots + src * 128 + rl);
                    return tot;
                }
                const uint32_t peer = xpeer;
                const int x = set * 2 + slot;
                float* mine = xv + x * 128 + rl;
                if (rl == 0) mbar_arrive_expect_tx(&xb[x], 128 * 4);
                st_async_f32(mapa_shared(smem_u32(mine), peer), part, mapa_shared(smem_u32(&xb[x]), peer));
                if (!mbar_wait(&xb[x], parity, EG2_DEV_TIMEOUT_GEMM, abort_flag)) {
                    ok = false;
                    return 0.f;
                }
                return part + *reinterpret_cast<volatile float*>(mine);
            };
            if constexpr (EPI == EPI_QKV_PAIR && WIDE) {
                // 16 warps: this warp takes chunk pairs c = 2 hw, 2 hw + 1 (columns 32 c.. and
                // 128 + 32 c.. of the CTA's half-head tile, in 16-pair sub-chunks). The head's sum of
                // squares: the quadrant's two half-warps meet first (as the sliding-layer WIDE form),
                // then the 8-warp form's exchange with the peer CTA (half 0 sends; both halves wait and
                // read; a slot is rewritten only after the peer has this CTA's next value, which half 0
                // sends after the next local meeting, i.e. after half 1 has read the slot).
                const QkvEpilogue& Q = epi.qkv;
                const int hidx = n0 / 512;
                int head, which;
                const float* w;
                bool rot;
                if (hidx < Q.nh) {
                    head = hidx, w = wsm, rot = true, which = 0;
                } else if (hidx < Q.nh + Q.nkv) {
                    head = hidx - Q.nh, w = wsm + BN, rot = true, which = 1;
                } else {
                    head = hidx - Q.nh - Q.nkv, w = nullptr, rot = false, which = 2;
                }
                float ss = 0.f;
#pragma unroll 1
                for (int cc = 0; cc < 2; cc++) {
                    const int c = 2 * hw + cc;
                    uint32_t r0[32], r1[32];
                    tmem_ld32(tbase + c * 32, r0);
                    tmem_ld32(tbase + 128 + c * 32, r1);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        ss = fmaf(__uint_as_float(r0[j]), __uint_as_float(r0[j]), ss);
                        ss = fmaf(__uint_as_float(r1[j]), __uint_as_float(r1[j]), ss);
                    }
                }
                {
                    float* xvl = reinterpret_cast<float*>(smem + Cfg::OFF_W + Cfg::XW_OFF) + (set * 4 + e) * 128 + (xq & 1) * 64;
                    uint64_t* xbl = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_W + Cfg::XWB_OFF) + (set * 4 + e) * 2 + (xq & 1);
                    xvl[hw * 32 + lane] = ss;
                    mbar_arrive(xbl);
                    if (!mbar_wait(xbl, (xq >> 1) & 1, EG2_DEV_TIMEOUT_GEMM, abort_flag)) break;
                    ss += *reinterpret_cast<volatile float*>(xvl + (hw ^ 1) * 32 + lane);
                    xq++;
                }
                float tot;
                {
                    float* xv = reinterpret_cast<float*>(smem + Cfg::OFF_W + Cfg::X_OFF);  // [set][slot][128]
                    uint64_t* xb = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_W + Cfg::XB_OFF);
                    const int rl = 32 * e + lane, x = set * 2 + (k & 1);
                    float* mine = xv + x * 128 + rl;
                    if (hw == 0) {
                        if (rl == 0) mbar_arrive_expect_tx(&xb[x], 128 * 4);
                        st_async_f32(mapa_shared(smem_u32(mine), crank ^ 1u), ss, mapa_shared(smem_u32(&xb[x]), crank ^ 1u));
                    }
                    if (!mbar_wait(&xb[x], (k >> 1) & 1, EG2_DEV_TIMEOUT_GEMM, abort_flag)) break;
                    tot = ss + *reinterpret_cast<volatile float*>(mine);
                }
                const float inv = 1.0f / sqrtf(tot / 512.f + Q.eps);
                const float* invs = wsm + 2 * BN;
                const int col1 = head * 512 + 128 * (int)crank, col2 = col1 + 256;
                const bool live = row < M;
                const float pf = (rot && live) ? (float)(Q.pos ? Q.pos[(long)row * Q.pos_stride] : row) : 0.f;
                const uint32_t sw32 = (uint32_t)((lane >> 2) & 1);
#pragma unroll 1
                for (int sc = 0; sc < 4; sc++) {
                    const int p = 64 * hw + 16 * sc;  // first pair (tile column) of the sub-chunk
                    float x1[16], x2[16];
                    {
                        uint32_t a[16], b[16];
                        tmem_ld16(tbase + p, a);
                        tmem_ld16(tbase + 128 + p, b);
                        tmem_ld_wait();
#pragma unroll
                        for (int t = 0; t < 16; t++) {
                            x1[t] = __uint_as_float(a[t]) * inv;
                            x2[t] = __uint_as_float(b[t]) * inv;
                        }
                    }
                    if (rot) {
#pragma unroll
                        for (int t = 0; t < 16; t++) {
                            const float a1 = x1[t] * w[p + t], a2 = x2[t] * w[128 + p + t];
                            float sj, cj;
                            sincos_reduced(pf * invs[p + t], sj, cj);
                            x1[t] = a1 * cj - a2 * sj;
                            x2[t] = a2 * cj + a1 * sj;
                        }
                    }
                    // Both 16-column pieces into the two 1 KB halves of slot nst % 2, one fence and group.
                    uint32_t p1[8], p2[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        p1[j] = bf16x2_bits(x1[2 * j], x1[2 * j + 1]);
                        p2[j] = bf16x2_bits(x2[2 * j], x2[2 * j + 1]);
                    }
                    uint8_t* buf = stage + (nst & 1) * 2048;
                    if (lane == 0) bulk_wait_read<1>();
                    __syncwarp();
#pragma unroll
                    for (int j = 0; j < 2; j++) {
                        *reinterpret_cast<uint4*>(buf + lane * 32 + ((j ^ sw32) << 4)) =
                            make_uint4(p1[4 * j], p1[4 * j + 1], p1[4 * j + 2], p1[4 * j + 3]);
                        *reinterpret_cast<uint4*>(buf + 1024 + lane * 32 + ((j ^ sw32) << 4)) =
                            make_uint4(p2[4 * j], p2[4 * j + 1], p2[4 * j + 2], p2[4 * j + 3]);
                    }
                    fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&em.m[which], buf, col1 + p, row0);
                        tma_store_2d(&em.m[which], buf + 1024, col2 + p, row0);
                        bulk_commit();
                    }
                    nst++;
                }
            } else if constexpr (EPI == EPI_QKV_PAIR) {
                // One head per 512-column group; as EPI_QKV (rowops.cu qkv_post_kernel arithmetic) with
                // the head's sum of squares completed by the exchange (slots alternate by tile parity).
                const QkvEpilogue& Q = epi.qkv;
                const int hidx = n0 / 512;
                TOut* base;
                int nheads, head;
                const float* w;
                bool rot;
                if (hidx < Q.nh) {
                    base = (TOut*)Q.q, nheads = Q.nh, head = hidx, w = wsm, rot = true;
                } else if (hidx < Q.nh + Q.nkv) {
                    base = (TOut*)Q.k, nheads = Q.nkv, head = hidx - Q.nh, w = wsm + BN, rot = true;
                } else {
                    base = (TOut*)Q.v, nheads = Q.nkv, head = hidx - Q.nh - Q.nkv, w = nullptr, rot = false;
                }
                float ss = 0.f;
#pragma unroll 1
                for (int c = 0; c < BN / 32; c += 2) {
                    uint32_t r0[32], r1[32];
                    tmem_ld32(tbase + c * 32, r0);
                    tmem_ld32(tbase + c * 32 + 32, r1);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        ss = fmaf(__uint_as_float(r0[j]), __uint_as_float(r0[j]), ss);
                        ss = fmaf(__uint_as_float(r1[j]), __uint_as_float(r1[j]), ss);
                    }
                }
                const float inv = 1.0f / sqrtf(exchange(ss, k & 1, (k >> 1) & 1) / 512.f + Q.eps);
                if (!ok) break;
                const float* invs = wsm + 2 * BN;
                const long ldo = (long)nheads * 512;
                const long col1 = (long)head * 512 + 128 * crank, col2 = col1 + 256;
                const bool live = row < M;
                const float pf = live ? (float)(Q.pos ? Q.pos[(long)row * Q.pos_stride] : row) : 0.f;
#pragma unroll 1
                for (int c = 0; c < 4; c++) {
                    float x1[32], x2[32];
                    {
                        uint32_t a[32], b[32];
                        tmem_ld32(tbase + c * 32, a);
                        tmem_ld32(tbase + 128 + c * 32, b);
                        tmem_ld_wait();
#pragma unroll
                        for (int t = 0; t < 32; t++) {
                            x1[t] = __uint_as_float(a[t]) * inv;
                            x2[t] = __uint_as_float(b[t]) * inv;
                        }
                    }
                    if (rot) {
#pragma unroll
                        for (int t = 0; t < 32; t++) {
                            const float a1 = x1[t] * w[c * 32 + t], a2 = x2[t] * w[128 + c * 32 + t];
                            float sj, cj;
                            sincos_reduced(pf * invs[c * 32 + t], sj, cj);
                            x1[t] = a1 * cj - a2 * sj;
                            x2[t] = a2 * cj + a1 * sj;
                        }
                    }
                    if constexpr (TIO) {
                        const int which = hidx < Q.nh ? 0 : hidx < Q.nh + Q.nkv ? 1 : 2;
                        tio_store32(&em.m[which], stage, nst++, x1, (int)col1 + c * 32, row0);
                        tio_store32(&em.m[which], stage, nst++, x2, (int)col2 + c * 32, row0);
                    } else {
                        warp_store32<TOut>(base, ldo, row0, M, col1 + c * 32, x1, stage);
                        warp_store32<TOut>(base, ldo, row0, M, col2 + c * 32, x2, stage);
                    }
                }
            } else if constexpr (DUAL) {
                // This layer's PLE slice p (second accumulator, BN columns after the gate g): the row
                // sums of squares of this CTA's 128 columns of p * scale go to the three other CTAs of
                // the cluster (st.async into each peer's slot [set][parity][this rank]); every CTA adds
                // the four partials in rank order, so all quarters of a row use the same norm. The slot
                // alternates with the set's tile parity, which is also the handshake (a peer writes this
                // set's slot for tile k + 2 only after it has this CTA's value for tile k + 1, sent after
                // this tile's slot was read here). Then out = bf16(gelu(g) * (p * scale * inv * w)): the
                // arithmetic of EPI_GROUP_NORM's stored value times the PLE-gate epilogue's GELU.
                const float* w1s = wsm;
                float ss = 0.f;
#pragma unroll 1
                for (int c = 0; c < BN / 32; c += 2) {
                    uint32_t r0[32], r1[32];
                    tmem_ld32(tbase + BN + c * 32, r0);
                    tmem_ld32(tbase + BN + c * 32 + 32, r1);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        const float a = __uint_as_float(r0[j]) * epi.scale, b = __uint_as_float(r1[j]) * epi.scale;
                        ss = fmaf(a, a, ss);
                        ss = fmaf(b, b, ss);
                    }
                }
                float inv;
                {
                    float* xv = reinterpret_cast<float*>(smem + Cfg::OFF_W + Cfg::X_OFF);     // [set][slot][src][128]
                    uint64_t* xb = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_W + Cfg::XB_OFF);  // [set][slot]
                    const int rl = 32 * e + lane;
                    const int x = set * 2 + (k & 1);
                    float* slots = xv + x * 4 * 128;
                    if (rl == 0) mbar_arrive_expect_tx(&xb[x], 3 * 128 * 4);
#pragma unroll
                    for (uint32_t pr = 0; pr < 4; pr++)
                        if (pr != crank)
                            st_async_f32(mapa_shared(smem_u32(slots + crank * 128 + rl), pr), ss,
                                         mapa_shared(smem_u32(&xb[x]), pr));
                    if (!mbar_wait(&xb[x], (k >> 1) & 1, EG2_DEV_TIMEOUT_GEMM, abort_flag)) {
                        ok = false;
                        break;
                    }
                    float tot = 0.f;
#pragma unroll
                    for (int src = 0; src < 4; src++)
                        tot += (src == (int)crank) ? ss : *reinterpret_cast<volatile float*>(slots + src * 128 + rl);
                    inv = 1.0f / sqrtf(tot / 512.f + epi.an.eps);
                }
                // 16-column chunks, bf16 through the slots (32-byte swizzle: row r's 16-byte unit j at
                // r * 32 + 16 * (j ^ ((r >> 2) & 1))) and out by TMA store.
                const uint32_t sw32 = (uint32_t)((lane >> 2) & 1);
#pragma unroll 1
                for (int c = 0; c < BN / 16; c++) {
                    uint32_t g[16], pv[16];
                    tmem_ld16(tbase + c * 16, g);
                    tmem_ld16(tbase + BN + c * 16, pv);
                    tmem_ld_wait();
                    uint32_t pk[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const float e0 = __uint_as_float(pv[2 * j]) * epi.scale * inv * w1s[c * 16 + 2 * j];
                        const float e1 = __uint_as_float(pv[2 * j + 1]) * epi.scale * inv * w1s[c * 16 + 2 * j + 1];
                        pk[j] = bf16x2_bits(gelu_fast(__uint_as_float(g[2 * j])) * e0, gelu_fast(__uint_as_float(g[2 * j + 1])) * e1);
                    }
                    uint8_t* slotp = stage + (nst & 3) * 2048;
                    if (lane == 0) bulk_wait_read<3>();  // the slot's previous store is read out
                    __syncwarp();
#pragma unroll
                    for (int j = 0; j < 2; j++)
                        *reinterpret_cast<uint4*>(slotp + lane * 32 + ((j ^ sw32) << 4)) =
                            make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
                    fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&em.m[0], slotp, n0 + 16 * c, row0);
                        bulk_commit();
                    }
                    nst++;
                }
            } else if constexpr (EPI == EPI_GROUP_NORM) {
                // One exchange per tile; the slot alternates with the tile's parity, which is also the
                // handshake: the peer writes this set's slot for tile k + 2 only after it has this CTA's
                // value for tile k + 1, sent after this tile's value was read here.
                const float* w1s = wsm;
                float ss = 0.f;
#pragma unroll 1
                for (int c = 0; c < BN / 32; c += 2) {
                    uint32_t r0[32], r1[32];
                    tmem_ld32(tbase + c * 32, r0);
                    tmem_ld32(tbase + c * 32 + 32, r1);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        const float a = __uint_as_float(r0[j]) * epi.scale, b = __uint_as_float(r1[j]) * epi.scale;
                        ss = fmaf(a, a, ss);
                        ss = fmaf(b, b, ss);
                    }
                }
                const float inv = 1.0f / sqrtf(exchange(ss, k & 1, (k >> 1) & 1) / 512.f + epi.an.eps);
                if (!ok) break;
                if constexpr (TIO) {
                    // f32 output in 16-column chunks through the slots (64-byte swizzle), by TMA store.
                    const uint32_t sw = (uint32_t)((lane >> 1) & 3);
#pragma unroll 1
                    for (int c = 0; c < BN / 16; c++) {
                        uint32_t r[16];
                        tmem_ld16(tbase + c * 16, r);
                        tmem_ld_wait();
                        float v[16];
#pragma unroll
                        for (int j = 0; j < 16; j++) v[j] = __uint_as_float(r[j]) * epi.scale * inv * w1s[c * 16 + j];
                        uint8_t* slot = stage + (nst & 3) * 2048;
                        if (lane == 0) bulk_wait_read<3>();  // the slot's previous store is read out
                        __syncwarp();
#pragma unroll
                        for (int j = 0; j < 4; j++)
                            *reinterpret_cast<float4*>(slot + lane * 64 + ((j ^ sw) << 4)) =
                                make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                        fence_proxy_async();
                        __syncwarp();
                        if (lane == 0) {
                            tma_store_2d(&em.m[0], slot, n0 + 16 * c, row0);
                            bulk_commit();
                        }
                        nst++;
                    }
                } else {
#pragma unroll 1
                    for (int c = 0; c < BN / 32; c++) {
                        uint32_t r[32];
                        tmem_ld32(tbase + c * 32, r);
                        tmem_ld_wait();
                        float v[32];
#pragma unroll
                        for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]) * epi.scale * inv * w1s[c * 32 + j];
                        warp_store32<TOut>(out, epi.ldo, row0, M, n0 + c * 32, v, stage);
                    }
                }
            } else if constexpr (EPI == EPI_ADD_NORM) {
                static_assert(TIO, "the add-norm epilogue runs with TMA I/O");
                // Residual in 16-column chunks through this warp's four 2 KB slots (64-byte swizzle:
                // row r's 16-byte unit j at r * 64 + 16 * (j ^ ((r >> 1) & 3)), conflict-free for
                // lane = row). Chunk c is read, updated in place and stored back by TMA; the load of
                // chunk c + 3 goes into the slot of chunk c - 1 once that store has been read out.
                // h_new stays in TMEM; t (bf16, 32 columns = one slot per chunk) is written from it
                // after the second exchange (t = h_new when there is no second norm).
                const AddNormEpilogue& A = epi.an;
                const float* w1s = wsm;
                const float* w2s = wsm + BN;
                const uint32_t sw = (uint32_t)((lane >> 1) & 3);
                float ss = 0.f;
#pragma unroll 1
                for (int c = 0; c < BN / 32; c += 2) {
                    uint32_t r0[32], r1[32];
                    tmem_ld32(tbase + c * 32, r0);
                    tmem_ld32(tbase + c * 32 + 32, r1);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        ss = fmaf(__uint_as_float(r0[j]), __uint_as_float(r0[j]), ss);
                        ss = fmaf(__uint_as_float(r1[j]), __uint_as_float(r1[j]), ss);
                    }
                }
                const float inv1 = 1.0f / sqrtf(exchange(ss, 0, k & 1) / (float)(256 * NP) + A.eps);
                if (!ok) break;
                float ss2 = 0.f;
#pragma unroll 1
                for (int c = 0; c < BN / 16; c++) {
                    uint8_t* buf = stage + (c & 3) * 2048 + lane * 64;
                    if (!mbar_wait(&hb[c & 3], (c >> 2) & 1, EG2_DEV_TIMEOUT_GEMM, abort_flag)) {
                        ok = false;
                        break;
                    }
                    ld_used++;
                    float hv[16];
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const float4 x = *reinterpret_cast<const float4*>(buf + ((j ^ sw) << 4));
                        hv[4 * j] = x.x, hv[4 * j + 1] = x.y, hv[4 * j + 2] = x.z, hv[4 * j + 3] = x.w;
                    }
                    if (c + 3 < BN / 16) {
                        if (lane == 0) {
                            bulk_wait_read<0>();  // the store of chunk c - 1 (same slot) is read out
                            const int s3 = (c + 3) & 3;
                            mbar_arrive_expect_tx(&hb[s3], 2048);
                            tma_load_2d(stage + s3 * 2048, &em.m[0], &hb[s3], n0 + 16 * (c + 3), row0);
                        }
                        ld_issued++;
                    }
                    uint32_t r[16];
                    tmem_ld16(tbase + c * 16, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        hv[j] = (hv[j] + __uint_as_float(r[j]) * inv1 * w1s[c * 16 + j]) * A.scalar;
                        ss2 = fmaf(hv[j], hv[j], ss2);
                        r[j] = __float_as_uint(hv[j]);
                    }
                    tmem_st16(tbase + c * 16, r);  // kept for t
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        *reinterpret_cast<float4*>(buf + ((j ^ sw) << 4)) =
                            make_float4(hv[4 * j], hv[4 * j + 1], hv[4 * j + 2], hv[4 * j + 3]);
                    fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&em.m[0], stage + (c & 3) * 2048, n0 + 16 * c, row0);
                        bulk_commit();
                    }
                }
                if (!ok) break;
                // The second exchange runs even without w2: it is also the handshake that keeps the
                // peer from writing this set's slot 0 for the next tile before it has been read here.
                tmem_st_wait();
                const float inv2 = 1.0f / sqrtf(exchange(ss2, 1, k & 1) / (float)(256 * NP) + A.eps);
                if (!ok) break;
#pragma unroll 1
                for (int c = 0; c < BN / 32; c++) {
                    uint32_t r[32];
                    tmem_ld32(tbase + c * 32, r);
                    tmem_ld_wait();
                    uint32_t pk[16];
                    if (A.w2) {
#pragma unroll
                        for (int j = 0; j < 16; j++)
                            pk[j] = bf16x2_bits(__uint_as_float(r[2 * j]) * inv2 * w2s[c * 32 + 2 * j],
                                              __uint_as_float(r[2 * j + 1]) * inv2 * w2s[c * 32 + 2 * j + 1]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; j++) pk[j] = bf16x2_bits(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
                    }
                    // Slot c % 4 was last the source of the 4th-newest store.
                    if (lane == 0) bulk_wait_read<3>();
                    __syncwarp();
                    uint8_t* buf = stage + (c & 3) * 2048 + lane * 64;
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        *reinterpret_cast<uint4*>(buf + ((j ^ sw) << 4)) =
                            make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
                    fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&em.m[1], stage + (c & 3) * 2048, n0 + 32 * c, row0);
                        bulk_commit();
                    }
                }
            } else if constexpr (EPI == EPI_QKV) {
                if constexpr (WIDE) {
                    float* xv = reinterpret_cast<float*>(smem + Cfg::OFF_W + Cfg::XW_OFF) + (set * 4 + e) * 128;
                    uint64_t* xbq = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_W + Cfg::XWB_OFF) + (set * 4 + e) * 2;
                    if (!epilogue_qkv256_wide(epi.qkv, tbase, row0, M, n0, stage, wsm, em, nst, hw, xv, xbq, xq,
                                              abort_flag))
                        break;
                } else {
                    epilogue_qkv<TOut, BN>(epi, tbase, row0, M, n0, stage, wsm);
                }
            } else if constexpr (EPI == EPI_PLE_GATE && TIO) {
                // GELU(gate) x ple[:, layer] in 16-column chunks: the inputs arrive by TMA in slot
                // c % 4 (f32, 64-byte swizzle), the bf16 result replaces them there (32-byte swizzle:
                // row r's 16-byte unit j at r * 32 + 16 * (j ^ ((r >> 2) & 1))) and leaves by TMA store;
                // the load of chunk c + 3 reuses the slot of chunk c - 1 once its store is read out.
                const uint32_t sw = (uint32_t)((lane >> 1) & 3), sw32 = (uint32_t)((lane >> 2) & 1);
#pragma unroll 1
                for (int c = 0; c < BN / 16; c++) {
                    uint8_t* slot = stage + (c & 3) * 2048;
                    if (!mbar_wait(&hb[c & 3], (c >> 2) & 1, EG2_DEV_TIMEOUT_GEMM, abort_flag)) {
                        ok = false;
                        break;
                    }
                    ld_used++;
                    float v[16];
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const float4 x = *reinterpret_cast<const float4*>(slot + lane * 64 + ((j ^ sw) << 4));
                        v[4 * j] = x.x, v[4 * j + 1] = x.y, v[4 * j + 2] = x.z, v[4 * j + 3] = x.w;
                    }
                    if (c + 3 < BN / 16) {
                        if (lane == 0) {
                            bulk_wait_read<0>();  // the store of chunk c - 1 (same slot) is read out
                            const int s3 = (c + 3) & 3;
                            mbar_arrive_expect_tx(&hb[s3], 2048);
                            tma_load_2d(stage + s3 * 2048, &em.m[1], &hb[s3], n0 + 16 * (c + 3), row0);
                        }
                        ld_issued++;
                    }
                    uint32_t r[16];
                    tmem_ld16(tbase + c * 16, r);
                    tmem_ld_wait();
                    uint32_t pk[8];
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        pk[j] = bf16x2_bits(gelu_fast(__uint_as_float(r[2 * j])) * v[2 * j],
                                            gelu_fast(__uint_as_float(r[2 * j + 1])) * v[2 * j + 1]);
                    __syncwarp();  // every lane has read its inputs from the slot
#pragma unroll
                    for (int j = 0; j < 2; j++)
                        *reinterpret_cast<uint4*>(slot + lane * 32 + ((j ^ sw32) << 4)) =
                            make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
                    fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&em.m[0], slot, n0 + 16 * c, row0);
                        bulk_commit();
                    }
                }
                if (!ok) break;
            } else if constexpr (EPI == EPI_PLE_GATE) {
                // GELU(gate) x ple[:, layer]: the per-layer inputs are read as coalesced 32 x 32 chunks
                // (4 whole 128-byte row segments per load instruction), one chunk ahead of their use.
                const float* pl = epi.aux + epi.aux_off;
                uint4 pa[8], pb[8];
                auto chunk = [&](int c, const uint4(&cur)[8]) {
                    float v[32];
                    warp_load32_finish(cur, v, stage);
                    uint32_t r[32];
                    tmem_ld32(tbase + c * 32, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 32; j++) v[j] = gelu_fast(__uint_as_float(r[j])) * v[j];
                    warp_store32<TOut>(out, epi.ldo, row0, M, n0 + c * 32, v, stage);
                };
                warp_load32_issue(pl, epi.aux_ld, row0, M, n0, pa);
#pragma unroll 1
                for (int c = 0; c < BN / 32; c += 2) {
                    warp_load32_issue(pl, epi.aux_ld, row0, M, n0 + (c + 1) * 32, pb);
                    chunk(c, pa);
                    if (c + 2 < BN / 32) warp_load32_issue(pl, epi.aux_ld, row0, M, n0 + (c + 2) * 32, pa);
                    chunk(c + 1, pb);
                }
            } else if constexpr (EPI == EPI_GELU_GU) {
                // Tile columns [0, BN/2) are gate features, [BN/2, BN) the matching up features.
#pragma unroll 1
                for (int c = 0; c < BN / 64; c++) {
                    float v[32];
                    {
                        uint32_t g[32], u[32];
                        tmem_ld32(tbase + c * 32, g);
                        tmem_ld32(tbase + BN / 2 + c * 32, u);
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 32; j++) v[j] = gelu_fast(__uint_as_float(g[j])) * __uint_as_float(u[j]);
                    }
                    if constexpr (TIO)
                        tio_store32(&em.m[0], stage, nst++, v, n0 / 2 + c * 32, row0);
                    else
                        warp_store32<TOut>(out, epi.ldo, row0, M, n0 / 2 + c * 32, v, stage);
                }
            } else {
                TOut* dst = out + (S > 1 ? (long)(tile % S) * epi.split_stride : 0L);  // K split: slice's partial
#pragma unroll 1
                for (int c = 0; c < BN / 32; c++) {
                    float v[32];
                    {
                        uint32_t r[32];
                        tmem_ld32(tbase + c * 32, r);
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
                    }
#pragma unroll
                    for (int j = 0; j < 32; j++) v[j] *= epi.scale;
                    warp_store32<TOut>(dst, epi.ldo, row0, M, n0 + c * 32, v, stage);
                }
            }
            tc_fence_before();
            if (!PAIR || lead)
                mbar_arrive(&tempty[set]);
            else
                mbar_arrive_remote(mapa_shared(smem_u32(&tempty[set]), pair_base));
        }
        if constexpr (TIO) {
            // Every TMA store has completed and every residual load issued has landed (bounded, for
            // the error path) before the CTA's shared memory goes away.
            if (lane == 0) {
                bulk_wait_all();
                for (int g = ld_used; g < ld_issued; g++) mbar_drain(&hb[g & 3], (g >> 2) & 1, 20000000ull);
            }
            __syncwarp();
        }
    }
done:
    if constexpr (PAIR) {
        // Every pair MMA (written into both CTAs' TMEM) has completed before either CTA frees it.
        if (lead && warp == 1 && lane == 0) {
            mma_commit_pair(smem_u32(drain));
            mbar_wait(drain, 0, EG2_DEV_TIMEOUT_GEMM, nullptr);
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR) {
        cluster_sync();
        if (warp == 1) {
            tc_fence_after();
            tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
        }
    } else {
        if (warp == 1) {
            tc_fence_after();
            tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
        }
        // No CTA leaves while its peer may still write into its shared memory.
        if constexpr (CL) cluster_sync();
    }
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------

template <typename TIn, int BN, int EPI, typename TOut>
static int launch_tc(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K, const GemmEpilogue& epi,
                     cudaStream_t s) {
    using Cfg = GemmCfg<BN>;
    auto kern = gemm_tc_kernel<TIn, BN, EPI, TOut>;
    static bool attr_set = false;  // per instantiation; set once per process (all devices share it)
    if (!attr_set) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES) != cudaSuccess)
            return -3;
        attr_set = true;
    }
    const int tiles = ((M + GEMM_BM - 1) / GEMM_BM) * (N / BN) * (epi.ksplit > 1 ? epi.ksplit : 1);
    const int grid = tiles < num_sms() ? tiles : num_sms();
    const EpiMaps none = {};  // no TMA epilogue I/O here
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(GEMM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, ta, tb, none, M, N, K, epi) == cudaSuccess ? 0 : -3;
}

// Clusters of two CTAs (the cluster epilogues, and CTA-pair MMAs), or of four (a cluster epilogue on
// CTA-pair MMAs), as many as can be resident at once (the loop over tiles is persistent, so every
// launched cluster must run concurrently with the others).
template <int EPI, typename TOut, bool PAIR = false, bool TIO = false, bool WIDE = false, int BNT = 256, int NP = 2>
static int launch_cluster(const CUtensorMap& ta, const CUtensorMap& tb, const EpiMaps& em, int M, int N, int K,
                          const GemmEpilogue& epi, cudaStream_t s) {
    constexpr bool DUAL = EPI == EPI_PLE_FUSED;
    using Cfg = GemmCfg<BNT, PAIR, TIO, WIDE, DUAL, NP>;
    auto kern = gemm_tc_kernel<bf16_t, BNT, EPI, TOut, PAIR, TIO, WIDE, NP>;
    constexpr bool QUAD = PAIR && (EPI == EPI_ADD_NORM || EPI == EPI_GROUP_NORM);
    constexpr int CSIZE = (QUAD || DUAL) ? 4 : NP;
    static int max_clusters[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -3;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CSIZE;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.blockDim = dim3(gemm_threads(WIDE), 1, 1);
    cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;  // the occupancy query takes the cluster shape only
    if (!max_clusters[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES) != cudaSuccess)
            return -3;
        cfg.gridDim = dim3(CSIZE * num_sms(), 1, 1);
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) return -3;
        max_clusters[dev] = n;
    }
    const int tiles_m = (M + GEMM_BM - 1) / GEMM_BM;
    if (N % ((PAIR && !QUAD) ? 256 : 256 * NP)) return -1;
    const long tiles = QUAD ? (long)((tiles_m + 1) / 2) * (N / 512)
                       : PAIR ? (long)((tiles_m + 1) / 2) * (N / 256) * (epi.ksplit > 1 ? epi.ksplit : 1)
                              : (long)tiles_m * (N / (DUAL ? 512 : 256 * NP));
    const int clusters = tiles < max_clusters[dev] ? (int)tiles : max_clusters[dev];
    cfg.gridDim = dim3(CSIZE * clusters, 1, 1);
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, ta, tb, em, M, N, K, epi) == cudaSuccess ? 0 : -3;
}

// CTA-pair MMAs for the plain epilogues; EG2_GEMM_NO_PAIR=1 selects the single-CTA kernels instead
// (same results up to summation order: both accumulate K in the same 64-element blocks).
static bool gemm_pair_enabled() {
    static const bool on = [] {
        const char* e = getenv("EG2_GEMM_NO_PAIR");
        return !(e && e[0] == '1');
    }();
    return on;
}

// Measured neutral on B200 (64 x 2,208-token step, same box: down 7.54 vs 7.76 ms, o 5.72 vs 5.52, ple_proj
// 4.59 vs 4.31, at 1,511 vs 1,477 MHz): the add-norm epilogue, not the main loop's shared-memory
// traffic, sets these GEMMs' pace, and clusters of four leave some SMs without a cluster. Off by default;
// EG2_ADD_NORM_QUAD=1 selects it (read per call: the A/B test switches it in-process).
static bool quad_enabled() {
    const char* e = getenv("EG2_ADD_NORM_QUAD");
    return e && e[0] == '1';
}

bool qkv_pair_fusable(const QkvEpilogue& q) {
    return q.hd == 512 && q.part == 512 && q.nh > 0 && q.nkv > 0 && q.wq && q.wk && q.inv_freq;
}

bool qkv_fusable(const QkvEpilogue& q) {
    const int hd = q.hd, half = q.part / 2;
    if (hd <= 0 || hd % 32 || 256 % hd || q.part <= 0 || hd % q.part) return false;
    if ((q.nh * hd) % 256 || (q.nkv * hd) % 256) return false;
    return q.part == 32 || (half >= 32 && half % 32 == 0);
}

int gemm_tc(GemmKind kind, const void* A, long lda, const void* W, long ldw, int M, int N, int K,
            const GemmEpilogue& epi, cudaStream_t s) {
    if (M <= 0) return 0;
    constexpr int BN = 256;
    const bool tf32 = kind == GEMM_TF32;
    const int esize = tf32 ? 4 : 2;
    const int BK = 128 / esize;
    if (N % BN || K % BK || lda % (16 / esize) || ldw % (16 / esize)) return -1;
    if (epi.mode == EPI_QKV && !qkv_fusable(epi.qkv)) return -1;
    CUtensorMap ta, tb;
    const CUtensorMapDataType dt = tf32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    if (make_tmap_2d(&ta, dt, A, K, M, lda * esize, BK, GEMM_BM)) return -1;
    // bf16 store / GELU / PLE-gate / QKV epilogues run on CTA pairs (each CTA loads half of the
    // weight tile, BN / 2 rows); the cluster epilogues and TF32 on single-CTA MMAs.
    const bool pair = !tf32 && (epi.mode == EPI_STORE || epi.mode == EPI_GELU_GU || epi.mode == EPI_PLE_GATE ||
                                epi.mode == EPI_QKV) && gemm_pair_enabled();
    // The add-norm epilogue on CTA-pair MMAs (clusters of four, opt-in): each CTA streams half of the
    // weight tile (same results as the single-CTA main loop: both accumulate K in the same 64-element
    // blocks).
    const bool quad = !tf32 && epi.mode == EPI_ADD_NORM && N == 512 && quad_enabled();
    if (make_tmap_2d(&tb, dt, W, K, N, ldw * esize, BK, (pair || quad) ? BN / 2 : BN)) return -1;
    const EpiMaps none = {};
    // bf16 output tensor [M, cols] (row stride ld elements) as 32 x 32 TMA store boxes.
    auto out_map = [&](CUtensorMap* m, const void* base, long cols, long ld) {
        return make_tmap_2d(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, cols, M, ld * 2, 32, 32,
                            CU_TENSOR_MAP_SWIZZLE_64B);
    };
    // K split: EPI_STORE with f32 partials (bf16 on CTA pairs, TF32 on single CTAs).
    if (epi.ksplit > 1 && ((!pair && !tf32) || epi.mode != EPI_STORE || (!epi.out_f32 && !tf32) || (K / BK) % epi.ksplit))
        return -1;
    if (pair) {
        switch (epi.mode) {
            case EPI_STORE:
                return epi.out_f32 ? launch_cluster<EPI_STORE, float, true>(ta, tb, none, M, N, K, epi, s)
                                   : launch_cluster<EPI_STORE, bf16_t, true>(ta, tb, none, M, N, K, epi, s);
            case EPI_GELU_GU: {
                EpiMaps em = {};
                if (epi.ldo % 8 || out_map(&em.m[0], epi.out, N / 2, epi.ldo)) return -1;
                return launch_cluster<EPI_GELU_GU, bf16_t, true, true>(ta, tb, em, M, N, K, epi, s);
            }
            case EPI_PLE_GATE: {
                // Inputs and outputs through TMA (the epilogue is bound by its global I/O): [0] the
                // bf16 output in 16 x 32 boxes, [1] this layer's slice of the PLE tensor (f32).
                EpiMaps em = {};
                if (epi.ldo % 8 || epi.aux_ld % 4 || epi.aux_off % 4 ||
                    make_tmap_2d(&em.m[0], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, epi.out, N, M, epi.ldo * 2, 16, 32,
                                 CU_TENSOR_MAP_SWIZZLE_32B) ||
                    make_tmap_2d(&em.m[1], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, epi.aux + epi.aux_off, N, M, epi.aux_ld * 4,
                                 16, 32, CU_TENSOR_MAP_SWIZZLE_64B))
                    return -1;
                return launch_cluster<EPI_PLE_GATE, bf16_t, true, true>(ta, tb, em, M, N, K, epi, s);
            }
            case EPI_QKV: {
                const QkvEpilogue& q = epi.qkv;
                if (q.hd == 256 && q.part == 256) {
                    // q / k / v in 16 x 32 boxes (32-byte swizzle) for the WIDE epilogue's stores.
                    EpiMaps em = {};
                    auto qkv_map = [&](CUtensorMap* m, const void* base, long cols) {
                        return make_tmap_2d(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, cols, M, cols * 2, 16, 32,
                                            CU_TENSOR_MAP_SWIZZLE_32B);
                    };
                    if (qkv_map(&em.m[0], q.q, (long)q.nh * 256) || qkv_map(&em.m[1], q.k, (long)q.nkv * 256) ||
                        qkv_map(&em.m[2], q.v, (long)q.nkv * 256))
                        return -1;
                    return launch_cluster<EPI_QKV, bf16_t, true, true, true>(ta, tb, em, M, N, K, epi, s);
                }
                return launch_cluster<EPI_QKV, bf16_t, true>(ta, tb, none, M, N, K, epi, s);
            }
        }
        return -1;
    }
    if (!tf32) {
        switch (epi.mode) {
            case EPI_STORE:
                return epi.out_f32 ? launch_tc<bf16_t, BN, EPI_STORE, float>(ta, tb, M, N, K, epi, s)
                                   : launch_tc<bf16_t, BN, EPI_STORE, bf16_t>(ta, tb, M, N, K, epi, s);
            case EPI_GELU_GU:
                return launch_tc<bf16_t, BN, EPI_GELU_GU, bf16_t>(ta, tb, M, N, K, epi, s);
            case EPI_PLE_GATE:
                return launch_tc<bf16_t, BN, EPI_PLE_GATE, bf16_t>(ta, tb, M, N, K, epi, s);
            case EPI_QKV:
                return launch_tc<bf16_t, BN, EPI_QKV, bf16_t>(ta, tb, M, N, K, epi, s);
            case EPI_ADD_NORM:
            {
                // Rows of 512 (text: clusters of two CTAs) or 768 (vision: clusters of three).
                if ((N != 512 && N != 768) || !epi.an.h || !epi.an.w1 || !epi.out || epi.ldo % 8) return -1;
                // The epilogue's residual I/O goes through TMA (the main loop keeps 3 stages); measured
                // faster than the register path with 4 stages for the O, down and PLE projections.
                // Residual h: f32 [M, 512], 16 x 32 boxes; t: bf16 [M, 512] (row stride ldo), 32 x 32.
                EpiMaps em = {};
                if (make_tmap_2d(&em.m[0], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, epi.an.h, N, M, (uint64_t)N * 4, 16, 32,
                                 CU_TENSOR_MAP_SWIZZLE_64B) ||
                    out_map(&em.m[1], epi.out, N, epi.ldo))
                    return -1;
                if (N == 768) return launch_cluster<EPI_ADD_NORM, bf16_t, false, true, false, 256, 3>(ta, tb, em, M, N, K, epi, s);
                return quad ? launch_cluster<EPI_ADD_NORM, bf16_t, true, true>(ta, tb, em, M, N, K, epi, s)
                            : launch_cluster<EPI_ADD_NORM, bf16_t, false, true>(ta, tb, em, M, N, K, epi, s);
            }
            case EPI_GROUP_NORM: {
                if (N % 512 || !epi.an.w1 || !epi.out || epi.ldo % 4) return -1;
                // f32 output by TMA store, 16 x 32 boxes.
                EpiMaps em = {};
                if (make_tmap_2d(&em.m[0], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, epi.out, N, M, epi.ldo * 4, 16, 32,
                                 CU_TENSOR_MAP_SWIZZLE_64B))
                    return -1;
                return launch_cluster<EPI_GROUP_NORM, float, false, true>(ta, tb, em, M, N, K, epi, s);
            }
            case EPI_QKV_PAIR: {
                const QkvEpilogue& q = epi.qkv;
                if (!qkv_pair_fusable(q) || N != (q.nh + 2 * q.nkv) * 512) return -1;
                // q / k / v by TMA store, 16 x 32 boxes (32-byte swizzle) for the 16-warp epilogue.
                EpiMaps em = {};
                auto qkv_map = [&](CUtensorMap* m, const void* base, long cols) {
                    return make_tmap_2d(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, cols, M, cols * 2, 16, 32,
                                        CU_TENSOR_MAP_SWIZZLE_32B);
                };
                if (qkv_map(&em.m[0], q.q, (long)q.nh * 512) || qkv_map(&em.m[1], q.k, (long)q.nkv * 512) ||
                    qkv_map(&em.m[2], q.v, (long)q.nkv * 512))
                    return -1;
                return launch_cluster<EPI_QKV_PAIR, bf16_t, false, true, true>(ta, tb, em, M, N, K, epi, s);
            }
        }
    } else {
        if (epi.mode == EPI_QKV) return launch_tc<float, BN, EPI_QKV, float>(ta, tb, M, N, K, epi, s);
        if (epi.mode == EPI_ADD_NORM || epi.mode == EPI_GROUP_NORM || epi.mode == EPI_QKV_PAIR) return -1;  // bf16 only
        switch (epi.mode) {
            case EPI_STORE:
                return launch_tc<float, BN, EPI_STORE, float>(ta, tb, M, N, K, epi, s);
            case EPI_GELU_GU:
                return launch_tc<float, BN, EPI_GELU_GU, float>(ta, tb, M, N, K, epi, s);
            case EPI_PLE_GATE:
                return launch_tc<float, BN, EPI_PLE_GATE, float>(ta, tb, M, N, K, epi, s);
        }
    }
    return -1;
}

int gemm_ple_fused(const bf16_t* t, const bf16_t* x, const bf16_t* w_gate, const bf16_t* w_ple_all, int layer,
                   const float* norm_w, float scale, float eps, bf16_t* out, int M, cudaStream_t s) {
    if (M <= 0) return 0;
    if (!t || !x || !w_gate || !w_ple_all || !norm_w || !out || layer < 0) return -1;
    constexpr int P = 512, BNT = 128;
    const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUtensorMap ta, tb;
    EpiMaps em = {};
    // A operands [M, 512] in 64 x 128 boxes; weight rows in 64 x 128 boxes (one 128-column quarter);
    // the output in 16 x 32 boxes with the 32-byte swizzle of the epilogue's slots.
    if (make_tmap_2d(&ta, dt, t, P, M, P * 2, 64, GEMM_BM) || make_tmap_2d(&tb, dt, w_gate, P, P, P * 2, 64, BNT) ||
        make_tmap_2d(&em.m[0], dt, out, P, M, P * 2, 16, 32, CU_TENSOR_MAP_SWIZZLE_32B) ||
        make_tmap_2d(&em.m[1], dt, x, P, M, P * 2, 64, GEMM_BM) ||
        make_tmap_2d(&em.m[2], dt, w_ple_all, P, (uint64_t)(layer + 1) * P, P * 2, 64, BNT))
        return -1;
    GemmEpilogue e;
    e.mode = EPI_PLE_FUSED;
    e.out = out;
    e.ldo = P;
    e.aux_off = layer * P;
    e.scale = scale;
    e.an.w1 = norm_w;
    e.an.eps = eps;
    return launch_cluster<EPI_PLE_FUSED, bf16_t, false, true, false, BNT>(ta, tb, em, M, P, P, e, s);
}

}  // namespace eg2

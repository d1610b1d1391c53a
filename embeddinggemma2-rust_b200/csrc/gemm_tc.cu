// Projection GEMMs on the 5th-generation tensor cores: C[M, N] = A[M, K] . W[N, K]^T with both
// operands K-major (nn.Linear layout), fp32 accumulation in tensor memory.
//
// Replaces the reference's cuBLAS calls `Gpu::gemm_bf16` (src/gpu/mod.rs:600-630, cublasGemmEx
// bf16 -> f32 accumulate) and `Gpu::matmul_nt` in TF32 mode (src/gpu/mod.rs:554-577), plus the
// elementwise kernels that follow them: `gelu_mul_gu` (kernels.cu:239-246, fused as EPI_GELU_GU)
// and `ple_gate` (kernels.cu:294-299, fused as EPI_PLE_GATE).
//
// Structure (one CTA per SM, persistent over output tiles of 128 x BN):
//   warp 0      TMA producer: A tile [128 x 64 bf16] and W tile [BN x 64] per stage, 128 B swizzle
//   warp 1      TMEM allocation; lane 0 issues tcgen05.mma (M=128, N=BN, K=16) and commits
//   warps 2..5  epilogue: tcgen05.ld of the accumulator, fused math, stores to global memory
// Two TMEM accumulators (2 x BN columns) let the epilogue of tile i overlap the MMAs of tile i+1.
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
constexpr int GEMM_THREADS = 192;

template <int BN>
struct GemmCfg {
    static constexpr int A_BYTES = GEMM_BM * 128;
    static constexpr int B_BYTES = BN * 128;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = (BN == 256) ? 4 : 6;
    static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 256;
    static constexpr uint32_t TMEM_COLS = 2 * BN;
};

template <typename TOut>
EG2_DEV void store32(TOut* dst, const float (&v)[32]);
template <>
EG2_DEV void store32<bf16_t>(bf16_t* dst, const float (&v)[32]) {
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int q = 0; q < 4; q++)
        d[q] = make_uint4(pack_bf16x2(v[8 * q + 0], v[8 * q + 1]), pack_bf16x2(v[8 * q + 2], v[8 * q + 3]),
                          pack_bf16x2(v[8 * q + 4], v[8 * q + 5]), pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
}
template <>
EG2_DEV void store32<float>(float* dst, const float (&v)[32]) {
    float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int q = 0; q < 8; q++) d[q] = make_float4(v[4 * q + 0], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
}

template <typename TIn, int BN, int EPI, typename TOut>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N, int K,
                   GemmEpilogue epi) {
    using Cfg = GemmCfg<BN>;
    constexpr int BK = InTraits<TIn>::BK;
    constexpr int STAGES = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_m = (M + GEMM_BM - 1) / GEMM_BM, tiles_n = N / BN;
    const int num_tiles = tiles_m * tiles_n;
    const int kblocks = K / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 128);
        }
        *abort_flag = 0;
        fence_mbarrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
                const int m0 = (tile / tiles_n) * GEMM_BM, n0 = (tile % tiles_n) * BN;
                for (int kb = 0; kb < kblocks; kb++) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, EG2_DEV_TIMEOUT_GEMM, abort_flag)) goto done;
                    uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
                    tma_load_2d(sa, &tmA, &full[stage], kb * BK, m0);
                    tma_load_2d(sa + Cfg::A_BYTES, &tmB, &full[stage], kb * BK, n0);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc(GEMM_BM, BN, InTraits<TIn>::FMT);
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, local++) {
                const int acc = local & 1;
                const uint32_t acc_phase = (local >> 1) & 1;
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1, EG2_DEV_TIMEOUT_GEMM, abort_flag)) goto done;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0; kb < kblocks; kb++) {
                    if (!mbar_wait(&full[stage], phase, EG2_DEV_TIMEOUT_GEMM, abort_flag)) goto done;
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + stage * Cfg::STAGE_BYTES);
                    const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < 4; kk++) {
                        const uint64_t ad = umma_desc_sw128(sa + kk * 32, 16, 1024);
                        const uint64_t bd = umma_desc_sw128(sb + kk * 32, 16, 1024);
                        mma_bf16_or_tf32<TIn>(d_tmem, ad, bd, idesc, (kb | kk) != 0);
                    }
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
        const int e = warp & 3;  // TMEM lane quadrant this warp may access
        int local = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, local++) {
            const int acc = local & 1;
            const uint32_t acc_phase = (local >> 1) & 1;
            if (!mbar_wait(&tfull[acc], acc_phase, EG2_DEV_TIMEOUT_GEMM, abort_flag)) break;
            tc_fence_after();
            const int m0 = (tile / tiles_n) * GEMM_BM, n0 = (tile % tiles_n) * BN;
            const int row = m0 + 32 * e + lane;
            const uint32_t tbase = tmem_base + ((uint32_t)(32 * e) << 16) + acc * BN;
            if constexpr (EPI == EPI_GELU_GU) {
                // Tile columns [0, BN/2) are gate features, [BN/2, BN) the matching up features.
                TOut* out = reinterpret_cast<TOut*>(epi.out);
#pragma unroll 1
                for (int c = 0; c < BN / 64; c++) {
                    uint32_t g[32], u[32];
                    tmem_ld32(tbase + c * 32, g);
                    tmem_ld32(tbase + BN / 2 + c * 32, u);
                    tmem_ld_wait();
                    float v[32];
#pragma unroll
                    for (int j = 0; j < 32; j++) v[j] = gelu_tanh_f(__uint_as_float(g[j])) * __uint_as_float(u[j]);
                    if (row < M) store32<TOut>(out + (long)row * epi.ldo + n0 / 2 + c * 32, v);
                }
            } else {
                TOut* out = reinterpret_cast<TOut*>(epi.out);
#pragma unroll 1
                for (int c = 0; c < BN / 32; c++) {
                    uint32_t r[32];
                    tmem_ld32(tbase + c * 32, r);
                    tmem_ld_wait();
                    float v[32];
                    if constexpr (EPI == EPI_PLE_GATE) {
                        if (row < M) {
                            const float4* pl = reinterpret_cast<const float4*>(epi.aux + (long)row * epi.aux_ld + epi.aux_off + n0 + c * 32);
#pragma unroll
                            for (int q = 0; q < 8; q++) {
                                float4 p4 = pl[q];
                                v[4 * q + 0] = gelu_tanh_f(__uint_as_float(r[4 * q + 0])) * p4.x;
                                v[4 * q + 1] = gelu_tanh_f(__uint_as_float(r[4 * q + 1])) * p4.y;
                                v[4 * q + 2] = gelu_tanh_f(__uint_as_float(r[4 * q + 2])) * p4.z;
                                v[4 * q + 3] = gelu_tanh_f(__uint_as_float(r[4 * q + 3])) * p4.w;
                            }
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]) * epi.scale;
                    }
                    if (row < M) store32<TOut>(out + (long)row * epi.ldo + n0 + c * 32, v);
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
        }
    }
done:
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
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
    const int tiles = ((M + GEMM_BM - 1) / GEMM_BM) * (N / BN);
    const int grid = tiles < num_sms() ? tiles : num_sms();
    kern<<<grid, GEMM_THREADS, Cfg::SMEM_BYTES, s>>>(ta, tb, M, N, K, epi);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int gemm_tc(GemmKind kind, const void* A, long lda, const void* W, long ldw, int M, int N, int K,
            const GemmEpilogue& epi, cudaStream_t s) {
    if (M <= 0) return 0;
    constexpr int BN = 256;
    const bool tf32 = kind == GEMM_TF32;
    const int esize = tf32 ? 4 : 2;
    const int BK = 128 / esize;
    if (N % BN || K % BK || lda % (16 / esize) || ldw % (16 / esize)) return -1;
    CUtensorMap ta, tb;
    const CUtensorMapDataType dt = tf32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    if (make_tmap_2d(&ta, dt, A, K, M, lda * esize, BK, GEMM_BM) || make_tmap_2d(&tb, dt, W, K, N, ldw * esize, BK, BN))
        return -1;
    if (!tf32) {
        switch (epi.mode) {
            case EPI_STORE:
                return epi.out_f32 ? launch_tc<bf16_t, BN, EPI_STORE, float>(ta, tb, M, N, K, epi, s)
                                   : launch_tc<bf16_t, BN, EPI_STORE, bf16_t>(ta, tb, M, N, K, epi, s);
            case EPI_GELU_GU:
                return launch_tc<bf16_t, BN, EPI_GELU_GU, bf16_t>(ta, tb, M, N, K, epi, s);
            case EPI_PLE_GATE:
                return launch_tc<bf16_t, BN, EPI_PLE_GATE, bf16_t>(ta, tb, M, N, K, epi, s);
        }
    } else {
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

}  // namespace eg2

// CUDA-core kernels of the float32 precision path: the f32 GEMM and the f32 attention.
//
// The float32 profile (embeddings within 5e-6 of the CPU path) rules out tensor cores, so these
// run on the FMA pipes. They mirror `Gpu::matmul_nt` without TF32 (src/gpu/mod.rs:554-577) and
// the fp32 attention of src/ops.rs:364-444 (bidirectional, scale 1, inclusive window, block
// diagonal per sequence), with an online softmax instead of materialised score blocks.
#include "common.cuh"
#include "kernels.h"

namespace eg2 {

// out[M, N] = scale * A[M, K] . W[N, K]^T; 64 x 64 tiles, 256 threads, 4 x 4 outputs per thread.
__global__ void __launch_bounds__(256) gemm_f32_kernel(const float* __restrict__ A, long lda, const float* __restrict__ W,
                                                       long ldw, float* __restrict__ out, long ldo, int M, int N, int K,
                                                       float scale) {
    constexpr int BM = 64, BN = 64, BK = 16;
    __shared__ float As[BK][BM + 4];
    __shared__ float Bs[BK][BN + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += BK) {
        for (int i = threadIdx.x; i < BM * BK; i += 256) {
            const int r = i / BK, c = i % BK;
            const int gm = m0 + r, gk = k0 + c;
            As[c][r] = (gm < M && gk < K) ? A[(long)gm * lda + gk] : 0.f;
            const int gn = n0 + r;
            Bs[c][r] = (gn < N && gk < K) ? W[(long)gn * ldw + gk] : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; kk++) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; i++) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; j++) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int gm = m0 + ty * 4 + i;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int gn = n0 + tx * 4 + j;
            if (gn < N) out[(long)gm * ldo + gn] = acc[i][j] * scale;
        }
    }
}

int gemm_f32(const float* A, long lda, const float* W, long ldw, float* out, long ldo, int M, int N, int K, float scale,
             cudaStream_t s) {
    if (M <= 0 || N <= 0) return 0;
    dim3 grid((N + 63) / 64, (M + 63) / 64);
    gemm_f32_kernel<<<grid, 256, 0, s>>>(A, lda, W, ldw, out, ldo, M, N, K, scale);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// ---------------------------------------------------------------------------------------------
// One warp per (row, query head). Lane l holds channels l, l + 32, ... of q and of the output.
// seq_start / seq_len: per row, the first row and the length of its sequence (block diagonal).
template <typename T, int NV>
__global__ void attention_simt_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                                      T* __restrict__ out, const int* __restrict__ seq_start,
                                      const int* __restrict__ seq_len, long rows, int nh, int nkv, int hd, int window) {
    const long item = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= rows * nh) return;
    const long row = item / nh;
    const int h = (int)(item % nh);
    const int g = h / (nh / nkv);
    const int lane = threadIdx.x & 31;
    const long start = seq_start[row];
    const int len = seq_len[row];
    const int pos = (int)(row - start);
    int lo = 0, hi = len;
    if (window >= 0) {
        lo = pos > window ? pos - window : 0;
        hi = pos + window + 1 < len ? pos + window + 1 : len;
    }
    float qv[NV], acc[NV];
    const T* qr = q + (row * nh + h) * hd;
#pragma unroll
    for (int j = 0; j < NV; j++) {
        qv[j] = (lane + 32 * j < hd) ? ldf(qr, lane + 32 * j) : 0.f;
        acc[j] = 0.f;
    }
    // Keys in groups of up to KG: each group's K rows (then V rows) are loaded together, so a warp has KG
    // rows in flight instead of one (short sequences are latency-bound on these loads); the running max
    // and the rescale of l and acc are updated once per group.
    constexpr int KG = 4;
    float m = -INFINITY, l = 0.f;
    for (int key0 = lo; key0 < hi; key0 += KG) {
        const int nk = hi - key0 < KG ? hi - key0 : KG;
        float kv[KG][NV];
#pragma unroll
        for (int kk = 0; kk < KG; kk++) {
            const T* kr = k + ((start + key0 + kk) * nkv + g) * hd;
#pragma unroll
            for (int j = 0; j < NV; j++) kv[kk][j] = (kk < nk && lane + 32 * j < hd) ? ldf(kr, lane + 32 * j) : 0.f;
        }
        float sd[KG];
#pragma unroll
        for (int kk = 0; kk < KG; kk++) {
            sd[kk] = 0.f;
#pragma unroll
            for (int j = 0; j < NV; j++) sd[kk] = fmaf(qv[j], kv[kk][j], sd[kk]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int kk = 0; kk < KG; kk++) sd[kk] += __shfl_xor_sync(0xffffffffu, sd[kk], o);
        float mn = m;
#pragma unroll
        for (int kk = 0; kk < KG; kk++)
            if (kk < nk) mn = fmaxf(mn, sd[kk]);
        const float corr = expf(m - mn);
        float pk[KG];
        float psum = 0.f;
#pragma unroll
        for (int kk = 0; kk < KG; kk++) {
            pk[kk] = kk < nk ? expf(sd[kk] - mn) : 0.f;
            psum += pk[kk];
        }
        l = l * corr + psum;
#pragma unroll
        for (int kk = 0; kk < KG; kk++) {
            const T* vr = v + ((start + key0 + kk) * nkv + g) * hd;
#pragma unroll
            for (int j = 0; j < NV; j++) kv[kk][j] = (kk < nk && lane + 32 * j < hd) ? ldf(vr, lane + 32 * j) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < NV; j++) {
            float a = acc[j] * corr;
#pragma unroll
            for (int kk = 0; kk < KG; kk++) a = fmaf(pk[kk], kv[kk][j], a);
            acc[j] = a;
        }
        m = mn;
    }
    const float inv = 1.f / l;
    T* orow = out + (row * nh + h) * hd;
#pragma unroll
    for (int j = 0; j < NV; j++)
        if (lane + 32 * j < hd) stf(orow, lane + 32 * j, acc[j] * inv);
}

template <typename T>
int attention_simt(const T* q, const T* k, const T* v, T* out, const int* seq_start, const int* seq_len, long rows, int nh,
                   int nkv, int hd, int window, cudaStream_t s) {
    if (rows <= 0) return 0;
    if (nh % nkv || hd > 512) return -1;
    const int wpb = 4;
    const long items = rows * nh;
    const unsigned grid = (unsigned)((items + wpb - 1) / wpb);
    if (hd <= 64)
        attention_simt_kernel<T, 2><<<grid, 32 * wpb, 0, s>>>(q, k, v, out, seq_start, seq_len, rows, nh, nkv, hd, window);
    else if (hd <= 256)
        attention_simt_kernel<T, 8><<<grid, 32 * wpb, 0, s>>>(q, k, v, out, seq_start, seq_len, rows, nh, nkv, hd, window);
    else
        attention_simt_kernel<T, 16><<<grid, 32 * wpb, 0, s>>>(q, k, v, out, seq_start, seq_len, rows, nh, nkv, hd, window);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
template int attention_simt<float>(const float*, const float*, const float*, float*, const int*, const int*, long, int, int,
                                   int, int, cudaStream_t);
template int attention_simt<bf16_t>(const bf16_t*, const bf16_t*, const bf16_t*, bf16_t*, const int*, const int*, long,
                                    int, int, int, int, cudaStream_t);

}  // namespace eg2

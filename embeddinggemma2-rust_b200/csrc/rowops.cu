// Row-wise and elementwise kernels of the forward pass. All arithmetic is f32; storage is f32 or
// bf16 as the template parameters say. HBM-bound: one warp per row (dim 512 or 768 here), 16-byte
// vector loads, no shared-memory staging except where a row's elements are exchanged (RoPE).
//
// Reference semantics (paths inside the reference project):
//   rms_norm_rows   src/ops.rs:211-238 (`rms_norm`), with the PLE pre-scale of src/text.rs:147-149
//   add_norm        src/text.rs:203-230 (post-norm + residual (+ layer_scalar), then the next pre-norm);
//                   GPU counterpart kernels.cu:131-172 (`add_norm_row`)
//   qkv_post        src/text.rs:171-175, src/vision.rs:241-245, src/ops.rs:319-338;
//                   GPU counterpart kernels.cu:183-237
//   gelu_gu         src/text.rs:210-212; kernels.cu:239-246
//   ple_gate        src/text.rs:218-224; kernels.cu:294-299
//   pool_rows       src/model.rs:530-535 + :677-688 (mean and L2 in f64, Matryoshka cuts)
//   embed_gather    src/text.rs:53-64
//   vision_*        src/vision.rs:73-89, :140-163; kernels.cu:249-282
#include "common.cuh"
#include "kernels.h"

namespace eg2 {

// Row kernels: one warp per row; lane l owns the VPL = dim / 32 contiguous columns
// [l * VPL, (l + 1) * VPL), so every load and store is a 16-byte vector and a warp sweeps each row
// as one contiguous 2 KB (f32) / 1 KB (bf16) span.
template <int VPL>
EG2_DEV void ld_row(const float* p, float (&v)[VPL]) {
#pragma unroll
    for (int q = 0; q < VPL / 4; q++) {
        const float4 a = reinterpret_cast<const float4*>(p)[q];
        v[4 * q] = a.x, v[4 * q + 1] = a.y, v[4 * q + 2] = a.z, v[4 * q + 3] = a.w;
    }
}
template <int VPL>
EG2_DEV void ld_row(const bf16_t* p, float (&v)[VPL]) {
#pragma unroll
    for (int q = 0; q < VPL / 8; q++) {
        const uint4 a = reinterpret_cast<const uint4*>(p)[q];
        const uint32_t u[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            v[8 * q + 2 * i] = __uint_as_float(u[i] << 16);
            v[8 * q + 2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
        }
    }
}
template <int VPL>
EG2_DEV void st_row(float* p, const float (&v)[VPL]) {
#pragma unroll
    for (int q = 0; q < VPL / 4; q++)
        reinterpret_cast<float4*>(p)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
}
template <int VPL>
EG2_DEV void st_row(bf16_t* p, const float (&v)[VPL]) {
#pragma unroll
    for (int q = 0; q < VPL / 8; q++)
        reinterpret_cast<uint4*>(p)[q] =
            make_uint4(bf16x2_bits(v[8 * q], v[8 * q + 1]), bf16x2_bits(v[8 * q + 2], v[8 * q + 3]),
                       bf16x2_bits(v[8 * q + 4], v[8 * q + 5]), bf16x2_bits(v[8 * q + 6], v[8 * q + 7]));
}

// ---------------------------------------------------------------------------------------------
template <typename TO, int VPL>
__global__ void rms_norm_kernel(const float* __restrict__ x, TO* __restrict__ out, const float* __restrict__ w, long rows,
                                float eps, float pre) {
    // The next kernel (a GEMM launched as a programmatic dependent) may start its prologue and weight
    // loads now; it reads this kernel's output only after this kernel has completed.
    grid_dep_launch();
    const long row = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    constexpr int dim = 32 * VPL;
    const long base = row * dim + (threadIdx.x & 31) * VPL;
    float v[VPL];
    ld_row<VPL>(x + base, v);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        v[i] *= pre;
        ss = fmaf(v[i], v[i], ss);
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)dim + eps);
    if (w) {
        float wv[VPL];
        ld_row<VPL>(w + (threadIdx.x & 31) * VPL, wv);
#pragma unroll
        for (int i = 0; i < VPL; i++) v[i] = v[i] * inv * wv[i];
    } else {
#pragma unroll
        for (int i = 0; i < VPL; i++) v[i] *= inv;
    }
    st_row<VPL>(out + base, v);
}

template <typename TO>
int rms_norm_rows(const float* x, TO* out, const float* w, long rows, int dim, float eps, float pre, cudaStream_t s) {
    if (rows <= 0) return 0;
    const int wpb = 8;
    const unsigned grid = (unsigned)((rows + wpb - 1) / wpb);
    if (dim == 512)
        rms_norm_kernel<TO, 16><<<grid, 32 * wpb, 0, s>>>(x, out, w, rows, eps, pre);
    else if (dim == 768)
        rms_norm_kernel<TO, 24><<<grid, 32 * wpb, 0, s>>>(x, out, w, rows, eps, pre);
    else
        return -1;
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
template int rms_norm_rows<float>(const float*, float*, const float*, long, int, float, float, cudaStream_t);
template int rms_norm_rows<bf16_t>(const float*, bf16_t*, const float*, long, int, float, float, cudaStream_t);

int rms_norm_inplace(float* x, const float* w, long rows, int dim, float eps, float pre, cudaStream_t s) {
    return rms_norm_rows<float>(x, x, w, rows, dim, eps, pre, s);
}

// ---------------------------------------------------------------------------------------------
// o may be split into nsplit partial sums (K slices of the producing GEMM), o_stride elements apart,
// added in slice order.
template <typename TI, typename TT, int VPL>
__global__ void add_norm_kernel(float* __restrict__ h, const TI* __restrict__ o, const float* __restrict__ w1,
                                TT* __restrict__ t, const float* __restrict__ w2, long rows, float eps, float scalar,
                                int nsplit = 1, long o_stride = 0) {
    grid_dep_launch();  // as in rms_norm_kernel
    const long row = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    constexpr int dim = 32 * VPL;
    const int c0 = (threadIdx.x & 31) * VPL;
    const long base = row * dim + c0;
    float v[VPL], hv[VPL], wv[VPL];
    ld_row<VPL>(o + base, v);
    for (int sp = 1; sp < nsplit; sp++) {
        ld_row<VPL>(o + sp * o_stride + base, hv);
#pragma unroll
        for (int i = 0; i < VPL; i++) v[i] += hv[i];
    }
    ld_row<VPL>(h + base, hv);
    ld_row<VPL>(w1 + c0, wv);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; i++) ss = fmaf(v[i], v[i], ss);
    ss = warp_sum(ss);
    const float inv1 = 1.0f / sqrtf(ss / (float)dim + eps);
    float ss2 = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        hv[i] = (hv[i] + v[i] * inv1 * wv[i]) * scalar;
        ss2 = fmaf(hv[i], hv[i], ss2);
    }
    st_row<VPL>(h + base, hv);
    if (!t) return;
    if (w2) {
        ss2 = warp_sum(ss2);
        const float inv2 = 1.0f / sqrtf(ss2 / (float)dim + eps);
        ld_row<VPL>(w2 + c0, wv);
#pragma unroll
        for (int i = 0; i < VPL; i++) hv[i] = hv[i] * inv2 * wv[i];
    }
    st_row<VPL>(t + base, hv);
}

template <typename TI, typename TT>
int add_norm(float* h, const TI* o, const float* w1, TT* t, const float* w2, long rows, int dim, float eps, float scalar,
             cudaStream_t s) {
    if (rows <= 0) return 0;
    const int wpb = 8;
    const unsigned grid = (unsigned)((rows + wpb - 1) / wpb);
    if (dim == 512)
        add_norm_kernel<TI, TT, 16><<<grid, 32 * wpb, 0, s>>>(h, o, w1, t, w2, rows, eps, scalar);
    else if (dim == 768)
        add_norm_kernel<TI, TT, 24><<<grid, 32 * wpb, 0, s>>>(h, o, w1, t, w2, rows, eps, scalar);
    else
        return -1;
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
template <typename TT>
int add_norm_split(float* h, const float* o, int nsplit, long o_stride, const float* w1, TT* t, const float* w2,
                   long rows, int dim, float eps, float scalar, cudaStream_t s) {
    if (rows <= 0) return 0;
    if (dim != 512 || nsplit < 1) return -1;
    const int wpb = 8;
    const unsigned grid = (unsigned)((rows + wpb - 1) / wpb);
    add_norm_kernel<float, TT, 16><<<grid, 32 * wpb, 0, s>>>(h, o, w1, t, w2, rows, eps, scalar, nsplit, o_stride);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
template int add_norm_split<bf16_t>(float*, const float*, int, long, const float*, bf16_t*, const float*, long, int, float,
                                    float, cudaStream_t);
template int add_norm_split<float>(float*, const float*, int, long, const float*, float*, const float*, long, int, float,
                                   float, cudaStream_t);
// GELU(g) x ple[:, layer] for g given as nsplit f32 partial sums (K slices), summed in slice order;
// the same arithmetic as the PLE-gate GEMM epilogue (gelu_fast). Four columns per thread.
template <typename TO>
__global__ void ple_gate_split_kernel(const float* __restrict__ part, int nsplit, long stride,
                                      const float* __restrict__ ple, long ple_ld, int ple_off, TO* __restrict__ out,
                                      long rows, int p) {
    grid_dep_launch();  // as in rms_norm_kernel
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;  // 4-column group
    const int gpr = p / 4;
    if (i >= rows * gpr) return;
    const long r = i / gpr;
    const int c = (int)(i % gpr) * 4;
    float4 g = *reinterpret_cast<const float4*>(part + r * p + c);
    for (int sp = 1; sp < nsplit; sp++) {
        const float4 x = *reinterpret_cast<const float4*>(part + sp * stride + r * p + c);
        g.x += x.x, g.y += x.y, g.z += x.z, g.w += x.w;
    }
    const float4 e = *reinterpret_cast<const float4*>(ple + r * ple_ld + ple_off + c);
    if constexpr (sizeof(TO) == 2) {
        uint2 o;
        o.x = bf16x2_bits(gelu_fast(g.x) * e.x, gelu_fast(g.y) * e.y);
        o.y = bf16x2_bits(gelu_fast(g.z) * e.z, gelu_fast(g.w) * e.w);
        *reinterpret_cast<uint2*>(out + r * p + c) = o;
    } else {
        *reinterpret_cast<float4*>(out + r * p + c) =
            make_float4(gelu_fast(g.x) * e.x, gelu_fast(g.y) * e.y, gelu_fast(g.z) * e.z, gelu_fast(g.w) * e.w);
    }
}

template <typename TO>
int ple_gate_split(const float* part, int nsplit, long stride, const float* ple, long ple_ld, int ple_off, TO* out,
                   long rows, int p, cudaStream_t s) {
    if (rows <= 0) return 0;
    if (p % 4 || ple_ld % 4 || ple_off % 4 || nsplit < 1) return -1;
    const long n = rows * (p / 4);
    ple_gate_split_kernel<TO><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(part, nsplit, stride, ple, ple_ld, ple_off, out,
                                                                          rows, p);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
template int ple_gate_split<bf16_t>(const float*, int, long, const float*, long, int, bf16_t*, long, int, cudaStream_t);
template int ple_gate_split<float>(const float*, int, long, const float*, long, int, float*, long, int, cudaStream_t);
template int add_norm<float, float>(float*, const float*, const float*, float*, const float*, long, int, float, float, cudaStream_t);
template int add_norm<bf16_t, bf16_t>(float*, const bf16_t*, const float*, bf16_t*, const float*, long, int, float, float, cudaStream_t);
template int add_norm<float, bf16_t>(float*, const float*, const float*, bf16_t*, const float*, long, int, float, float, cudaStream_t);

// ---------------------------------------------------------------------------------------------
// One warp per (row, head slot) over [q heads | k heads | v heads]. The normalised head goes
// through shared memory so RoPE can pair element i with i + part/2 whatever the lane layout.
// Tables hold the unique half of the reference's duplicated-halves layout: entry
// [pos, pi * (part / 2) + j] is the angle of rotation part pi, frequency j; rope_w = hd / 2.
template <typename TI, typename TO>
__global__ void qkv_post_kernel(const TI* __restrict__ qkv, TO* __restrict__ q, TO* __restrict__ k, TO* __restrict__ v,
                                const float* __restrict__ wq, const float* __restrict__ wk, const float* __restrict__ cs,
                                const float* __restrict__ sn, int rope_w, const int* __restrict__ pos, long rows, int nh,
                                int nkv, int hd, int part, float eps, int nsplit = 1, long split_stride = 0) {
    extern __shared__ float sbuf[];
    const int S = nh + 2 * nkv;
    const long item = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= rows * S) return;
    const long row = item / S;
    const int slot = (int)(item % S);
    const int lane = threadIdx.x & 31;
    float* buf = sbuf + (threadIdx.x >> 5) * hd;
    const TI* src = qkv + row * (long)S * hd + (long)slot * hd;
    const float* w;
    TO* dst;
    bool rot;
    if (slot < nh) {
        dst = q + (row * nh + slot) * hd;
        w = wq;
        rot = true;
    } else if (slot < nh + nkv) {
        dst = k + (row * nkv + (slot - nh)) * hd;
        w = wk;
        rot = true;
    } else {
        dst = v + (row * nkv + (slot - nh - nkv)) * hd;
        w = nullptr;
        rot = false;
    }
    float ss = 0.f;
    if (nsplit == 1) {
        for (int i = lane; i < hd; i += 32) {
            const float x = ldf(src, i);
            buf[i] = x;
            ss = fmaf(x, x, ss);
        }
    } else {
        // K-split partials (at most 8), all loaded before they are added in slice order.
        for (int i = lane; i < hd; i += 32) {
            float pv[8];
#pragma unroll
            for (int sp = 0; sp < 8; sp++) pv[sp] = sp < nsplit ? ldf(src + sp * split_stride, i) : 0.f;
            float x = pv[0];
#pragma unroll
            for (int sp = 1; sp < 8; sp++)
                if (sp < nsplit) x += pv[sp];
            buf[i] = x;
            ss = fmaf(x, x, ss);
        }
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)hd + eps);
    for (int i = lane; i < hd; i += 32) {
        float n = buf[i] * inv;
        if (w) n *= w[i];
        buf[i] = n;
    }
    __syncwarp();
    if (!rot) {
        for (int i = lane; i < hd; i += 32) stf(dst, i, buf[i]);
        return;
    }
    const int half = part / 2;
    const long p = pos ? pos[row] : row;
    const float* c = cs + p * rope_w;
    const float* sv = sn + p * rope_w;
    for (int idx = lane; idx < hd / 2; idx += 32) {
        const int pi = idx / half, j = idx % half;
        const int b = pi * part;
        const float x1 = buf[b + j], x2 = buf[b + half + j];
        const float cj = c[pi * half + j], sj = sv[pi * half + j];
        stf(dst, b + j, x1 * cj - x2 * sj);
        stf(dst, b + half + j, x2 * cj + x1 * sj);
    }
}

template <typename TI, typename TO>
int qkv_post(const TI* qkv, TO* q, TO* k, TO* v, const float* wq, const float* wk, const float* cs, const float* sn,
             int rope_w, const int* pos, long rows, int nh, int nkv, int hd, int part, float eps, cudaStream_t s) {
    if (rows <= 0) return 0;
    if (hd % 32 || hd > 1024 || part <= 0 || hd % part || part % 2) return -1;
    const int wpb = 8;
    const long items = rows * (nh + 2 * nkv);
    qkv_post_kernel<TI, TO><<<(unsigned)((items + wpb - 1) / wpb), 32 * wpb, wpb * hd * sizeof(float), s>>>(
        qkv, q, k, v, wq, wk, cs, sn, rope_w, pos, rows, nh, nkv, hd, part, eps);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
// qkv given as nsplit f32 partial sums (K slices of the producing GEMM) split_stride elements apart.
int qkv_post_split(const float* qkv, int nsplit, long split_stride, float* q, float* k, float* v, const float* wq,
                   const float* wk, const float* cs, const float* sn, int rope_w, const int* pos, long rows, int nh,
                   int nkv, int hd, int part, float eps, cudaStream_t s) {
    if (rows <= 0) return 0;
    if (hd % 32 || hd > 1024 || part <= 0 || hd % part || part % 2 || nsplit < 1 || nsplit > 8) return -1;
    const int wpb = 8;
    const long items = rows * (nh + 2 * nkv);
    qkv_post_kernel<float, float><<<(unsigned)((items + wpb - 1) / wpb), 32 * wpb, wpb * hd * sizeof(float), s>>>(
        qkv, q, k, v, wq, wk, cs, sn, rope_w, pos, rows, nh, nkv, hd, part, eps, nsplit, split_stride);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
template int qkv_post<bf16_t, bf16_t>(const bf16_t*, bf16_t*, bf16_t*, bf16_t*, const float*, const float*, const float*,
                                      const float*, int, const int*, long, int, int, int, int, float, cudaStream_t);
template int qkv_post<float, float>(const float*, float*, float*, float*, const float*, const float*, const float*,
                                    const float*, int, const int*, long, int, int, int, int, float, cudaStream_t);

// ---------------------------------------------------------------------------------------------
// gate|up rows in the interleaved layout of EPI_GELU_GU: per 256 columns, 128 gate then 128 up.
template <typename TI, typename TO>
__global__ void gelu_gu_kernel(const TI* __restrict__ gu, TO* __restrict__ out, long rows, int ff) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * ff) return;
    const long r = i / ff;
    const int c = (int)(i % ff);
    const long base = r * 2L * ff + (c / 128) * 256 + (c % 128);
    stf(out, i, gelu_tanh_f(ldf(gu, base)) * ldf(gu, base + 128));
}
template <typename TI, typename TO>
int gelu_gu(const TI* gu, TO* out, long rows, int ff, cudaStream_t s) {
    if (rows <= 0) return 0;
    if (ff % 128) return -1;
    const long n = rows * ff;
    gelu_gu_kernel<TI, TO><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(gu, out, rows, ff);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
template int gelu_gu<float, float>(const float*, float*, long, int, cudaStream_t);

// gelu(gate) * up from nsplit f32 partial sums of the interleaved gate|up projection (stride apart),
// summed in slice order; gelu_fast, as the EPI_GELU_GU epilogue computes it.
__global__ void gelu_gu_split_kernel(const float* __restrict__ part, int nsplit, long stride, float* __restrict__ out,
                                     long rows, int ff) {
    grid_dep_launch();  // as in rms_norm_kernel
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * ff) return;
    const long r = i / ff;
    const int c = (int)(i % ff);
    const long base = r * 2L * ff + (c / 128) * 256 + (c % 128);
    float g = part[base], u = part[base + 128];
    for (int sp = 1; sp < nsplit; sp++) {
        g += part[sp * stride + base];
        u += part[sp * stride + base + 128];
    }
    out[i] = gelu_fast(g) * u;
}
int gelu_gu_split(const float* part, int nsplit, long stride, float* out, long rows, int ff, cudaStream_t s) {
    if (rows <= 0) return 0;
    if (ff % 128 || nsplit < 1) return -1;
    const long n = rows * ff;
    gelu_gu_split_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(part, nsplit, stride, out, rows, ff);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

template <typename TI, typename TO>
__global__ void ple_gate_kernel(const TI* __restrict__ g, TO* __restrict__ out, const float* __restrict__ ple, long rows,
                                int p, int n_layers, int layer) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * p) return;
    const long r = i / p;
    const int c = (int)(i % p);
    stf(out, i, gelu_tanh_f(ldf(g, i)) * ple[(r * n_layers + layer) * p + c]);
}
template <typename TI, typename TO>
int ple_gate(const TI* g, TO* out, const float* ple, long rows, int p, int n_layers, int layer, cudaStream_t s) {
    if (rows <= 0) return 0;
    const long n = rows * p;
    ple_gate_kernel<TI, TO><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(g, out, ple, rows, p, n_layers, layer);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
template int ple_gate<float, float>(const float*, float*, const float*, long, int, int, int, cudaStream_t);

// ---------------------------------------------------------------------------------------------
// Mean over a sequence's rows (f64 sums), L2 normalisation (f64) and Matryoshka cuts: for each
// sequence the output holds, back to back, the normalised first dims[d] components for each d.
// Two stages so that every SM works on long sequences: pool_partial_kernel sums chunks of
// POOL_CHUNK rows (block (s, ch), one float4 column group per thread) into partial[s][ch][dim];
// pool_final_kernel adds a sequence's chunks in order (deterministic) and normalises.
constexpr int POOL_CHUNK = 128;

__global__ void pool_partial_kernel(const float* __restrict__ x, const int* __restrict__ seq_start,
                                    const int* __restrict__ seq_len, int dim, int n_chunks, double* __restrict__ partial) {
    const int s = blockIdx.x, ch = blockIdx.y;
    const long r0 = seq_start[s];
    const int len = seq_len[s];
    const int a = ch * POOL_CHUNK, b = min(len, a + POOL_CHUNK);
    for (int c4 = threadIdx.x; c4 < dim / 4; c4 += blockDim.x) {
        double acc[4] = {0.0, 0.0, 0.0, 0.0};
        const float* col = x + (r0 + a) * dim + 4 * c4;
#pragma unroll 4
        for (int r = a; r < b; r++, col += dim) {
            const float4 v = *reinterpret_cast<const float4*>(col);
            acc[0] += (double)v.x, acc[1] += (double)v.y, acc[2] += (double)v.z, acc[3] += (double)v.w;
        }
        double* dst = partial + ((long)s * n_chunks + ch) * dim + 4 * c4;
        dst[0] = acc[0], dst[1] = acc[1], dst[2] = acc[2], dst[3] = acc[3];
    }
}

__global__ void pool_final_kernel(const double* __restrict__ partial, const int* __restrict__ seq_len, int dim,
                                  int n_chunks, const int* __restrict__ dims, int n_dims, int out_stride,
                                  float* __restrict__ out) {
    extern __shared__ double dsh[];  // dim means + 32 partials
    double* mean = dsh;
    double* part = dsh + dim;
    const int sidx = blockIdx.x;
    const int len = seq_len[sidx];
    const int used = (len + POOL_CHUNK - 1) / POOL_CHUNK;
    for (int c = threadIdx.x; c < dim; c += blockDim.x) {
        double acc = 0.0;
        for (int ch = 0; ch < used; ch++) acc += partial[((long)sidx * n_chunks + ch) * dim + c];
        mean[c] = (double)(float)(acc / (double)len);
    }
    __syncthreads();
    float* o = out + (long)sidx * out_stride;
    int off = 0;
    for (int d = 0; d < n_dims; d++) {
        const int nd = dims[d];
        double ss = 0.0;
        for (int c = threadIdx.x; c < nd; c += blockDim.x) ss += mean[c] * mean[c];
#pragma unroll
        for (int sh = 16; sh > 0; sh >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, sh);
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
        __syncthreads();
        double tot = 0.0;
        for (int wv = 0; wv < (int)(blockDim.x >> 5); wv++) tot += part[wv];
        const double norm = fmax(sqrt(tot), 1e-12);
        for (int c = threadIdx.x; c < nd; c += blockDim.x) o[off + c] = (float)(mean[c] / norm);
        __syncthreads();
        off += nd;
    }
}

int pool_scratch_doubles(int n_seq, int max_len, int dim) {
    return n_seq * ((max_len + POOL_CHUNK - 1) / POOL_CHUNK) * dim;
}

int pool_rows(const float* x, const int* seq_start, const int* seq_len, int n_seq, int max_len, int dim,
              const int* dims_dev, int n_dims, int out_stride, float* out, double* scratch, cudaStream_t s) {
    if (n_seq <= 0) return 0;
    if (dim % 4) return -1;
    const int n_chunks = (max_len + POOL_CHUNK - 1) / POOL_CHUNK;
    pool_partial_kernel<<<dim3(n_seq, n_chunks), 192, 0, s>>>(x, seq_start, seq_len, dim, n_chunks, scratch);
    pool_final_kernel<<<n_seq, 256, (dim + 32) * sizeof(double), s>>>(scratch, seq_len, dim, n_chunks, dims_dev, n_dims,
                                                                     out_stride, out);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// ---------------------------------------------------------------------------------------------
__global__ void embed_gather_kernel(const bf16_t* __restrict__ table, long vocab, int h, const uint32_t* __restrict__ ids,
                                    long n, float scale, float* __restrict__ out, int* bad) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * h) return;
    const long t = i / h;
    const int c = (int)(i % h);
    const uint32_t id = ids[t];
    if ((long)id >= vocab) {
        if (c == 0) atomicExch(bad, 1);
        out[i] = 0.f;
        return;
    }
    out[i] = bf16_to_f32(table[(long)id * h + c]) * scale;
}
int embed_gather(const bf16_t* table, long vocab, int h, const uint32_t* ids, long n, float scale, float* out, int* bad,
                 cudaStream_t s) {
    if (n <= 0) return 0;
    const long tot = n * h;
    embed_gather_kernel<<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(table, vocab, h, ids, n, scale, out, bad);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// The text pass's first three steps in one row kernel (bf16 contexts, 512-wide rows): the embedding
// gather times scale (f32 hidden), its bf16 copy (the PLE projection's input) and the first layer's
// pre-norm (bf16 t) -- the arithmetic of embed_gather_kernel, cast_kernel and rms_norm_kernel in turn,
// with one read of the table row instead of two more of hidden.
template <int VPL>
__global__ void embed_gather_norm_kernel(const bf16_t* __restrict__ table, long vocab, const uint32_t* __restrict__ ids,
                                         long n, float scale, float* __restrict__ hidden, bf16_t* __restrict__ xb,
                                         bf16_t* __restrict__ t, const float* __restrict__ w, float eps, int* bad) {
    grid_dep_launch();  // as in rms_norm_kernel
    const long row = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= n) return;
    constexpr int dim = 32 * VPL;
    const int lane = threadIdx.x & 31;
    const uint32_t id = ids[row];
    float v[VPL];
    if ((long)id >= vocab) {
        if (lane == 0) atomicExch(bad, 1);
#pragma unroll
        for (int i = 0; i < VPL; i++) v[i] = 0.f;
    } else {
        ld_row<VPL>(table + (long)id * dim + lane * VPL, v);
#pragma unroll
        for (int i = 0; i < VPL; i++) v[i] *= scale;
    }
    const long base = row * dim + lane * VPL;
    st_row<VPL>(hidden + base, v);
    st_row<VPL>(xb + base, v);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; i++) ss = fmaf(v[i], v[i], ss);
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)dim + eps);
    float wv[VPL];
    ld_row<VPL>(w + lane * VPL, wv);
#pragma unroll
    for (int i = 0; i < VPL; i++) v[i] = v[i] * inv * wv[i];
    st_row<VPL>(t + base, v);
}
int embed_gather_norm(const bf16_t* table, long vocab, int h, const uint32_t* ids, long n, float scale, float* hidden,
                      bf16_t* xb, bf16_t* t, const float* w, float eps, int* bad, cudaStream_t s) {
    if (n <= 0) return 0;
    if (h != 512) return -1;
    const int wpb = 8;
    embed_gather_norm_kernel<16><<<(unsigned)((n + wpb - 1) / wpb), 32 * wpb, 0, s>>>(table, vocab, ids, n, scale, hidden, xb,
                                                                                    t, w, eps, bad);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// Per-row metadata of a pass from its sequence offsets (off[s] = first row of sequence s, off[n_seq] =
// rows): the row's position in its sequence, the sequence's first row and its length -- what the
// host used to expand row by row and upload (12 bytes per row).
__global__ void row_meta_kernel(const int* __restrict__ off, int n_seq, long rows, int* __restrict__ pos,
                                int* __restrict__ st, int* __restrict__ ln) {
    const long r = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    int lo = 0, hi = n_seq - 1;  // the last s with off[s] <= r
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (off[mid] <= r) lo = mid;
        else hi = mid - 1;
    }
    const int s0 = off[lo];
    pos[r] = (int)(r - s0);
    st[r] = s0;
    ln[r] = off[lo + 1] - s0;
}

int row_meta(const int* off, int n_seq, long rows, int* pos, int* st, int* ln, cudaStream_t s) {
    if (rows <= 0 || n_seq <= 0) return 0;
    row_meta_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, s>>>(off, n_seq, rows, pos, st, ln);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

template <typename TO>
__global__ void cast_kernel(const float* __restrict__ x, TO* __restrict__ out, long n, float mul, float add) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) stf(out, i, (x[i] + add) * mul);
}
template <typename TO>
int cast_rows(const float* x, TO* out, long n, float mul, float add, cudaStream_t s) {
    if (n <= 0) return 0;
    cast_kernel<TO><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, out, n, mul, add);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
template int cast_rows<float>(const float*, float*, long, float, float, cudaStream_t);
template int cast_rows<bf16_t>(const float*, bf16_t*, long, float, float, cudaStream_t);

__global__ void widen_bf16_kernel(const bf16_t* __restrict__ x, float* __restrict__ out, long n) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = bf16_to_f32(x[i]);
}
int widen_bf16(const bf16_t* x, float* out, long n, cudaStream_t s) {
    if (n <= 0) return 0;
    widen_bf16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, out, n);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

__global__ void vision_pos_kernel(float* __restrict__ h, const float* __restrict__ table, const int* __restrict__ pos, long n,
                                  int hdim, int pe) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * hdim) return;
    const long t = i / hdim;
    const int c = (int)(i % hdim);
    h[i] += table[(long)pos[2 * t] * hdim + c] + table[((long)pe + pos[2 * t + 1]) * hdim + c];
}
int vision_add_positions(float* h, const float* table, const int* pos, long n, int hdim, int pe, cudaStream_t s) {
    if (n <= 0) return 0;
    vision_pos_kernel<<<(unsigned)((n * hdim + 255) / 256), 256, 0, s>>>(h, table, pos, n, hdim, pe);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

__global__ void vision_pool_kernel(const float* __restrict__ x, float* __restrict__ out, int gh, int gw, int hdim, int k,
                                   float root) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const int ow = gw / k;
    const long n = (long)(gh / k) * ow * hdim;
    if (i >= n) return;
    const long o = i / hdim;
    const int c = (int)(i % hdim);
    const int oy = (int)(o / ow), ox = (int)(o % ow);
    float acc = 0.f;
    for (int dy = 0; dy < k; dy++)
        for (int dx = 0; dx < k; dx++) acc += x[((long)(oy * k + dy) * gw + ox * k + dx) * hdim + c];
    out[i] = (acc / (float)(k * k)) * root;
}
int vision_pool(const float* x, float* out, int gh, int gw, int hdim, int k, float root, cudaStream_t s) {
    const long n = (long)(gh / k) * (gw / k) * hdim;
    if (n <= 0) return 0;
    vision_pool_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, out, gh, gw, hdim, k, root);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace eg2

namespace eg2 {
template int qkv_post<float, bf16_t>(const float*, bf16_t*, bf16_t*, bf16_t*, const float*, const float*, const float*,
                                     const float*, int, const int*, long, int, int, int, int, float, cudaStream_t);
}  // namespace eg2

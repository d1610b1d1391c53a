// The reference engine's own CUDA backend for the text backbone, timed on sm_100 as a baseline.
//
// The reference drives its GPU kernels from Rust (cudarc): cuBLAS GemmEx for every projection and the
// NVRTC-compiled kernels of src/gpu/kernels.cu + kernels_sm80.cu for the rest. Rust is not available
// here, so this file restates that driver in C++: the bf16 launch sequence of GpuText::enqueue
// (src/gpu/text.rs:350-433), with the launch geometry and arguments of the Gpu helpers it calls
// (src/gpu/mod.rs: gemm_bf16 :605-631, matmul_nt_bf16 :584-598, rms_norm_impl :674-691, rms_norm_act
// :693-709, add_norm_act :755-794, qkv_post_from :843-865, gelu_mul_strided :1025-1033, ple_gate_act
// :991-1004, flash_launch :1346-1355, flash_d512_launch :1372-1386) and the host-side RoPE tables of
// ops::rope_tables (src/ops.rs:293-314). The kernels themselves are the reference's, compiled by nvcc from
// their own files (the Makefile passes their paths; defines as src/gpu/mod.rs:299-300: EG_BF16 and
// FLASH_D512_BK = 32), and the GEMMs are cuBLAS, as in the reference. One pass = one call of
// GpuText::forward_packed for sequences longer than 256 tokens (no CUDA graph, attention per sequence).
//
// This is a measurement harness, not part of the library: nothing in the package links it.
#undef INFINITY
#define EG_BF16
#define FLASH_D512_BK 32
#include REF_KERNELS
#include REF_KERNELS_SM80

#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

namespace refgpu {

constexpr float NEG_INF = -__builtin_huge_valf();
constexpr float POS_INF = __builtin_huge_valf();
constexpr int FLASH_D512_SMEM = 2 * FLASH_D512_BK * 512 * 2 + 8 * 16 * FLASH_D512_BK * 4;

// Threads of a row reduction over `dim` elements (src/gpu/mod.rs:253-255).
static unsigned norm_threads(int dim) { return dim >= 1024 ? 256 : dim >= 256 ? 128 : 64; }
static unsigned blocks_1d(long long n, int per = 256) { return (unsigned)((n + per - 1) / per); }

struct Layer {
    int hd, nkv, window;  // window < 0: global
    double theta;
    uint16_t *qkv, *o, *gu, *down, *pg, *pp;  // bf16 [out, in]; qkv = q|k|v rows, gu = gate|up rows
    float *input_ln, *post_attn_ln, *pre_ff_ln, *post_ff_ln, *q_norm, *k_norm, *ple_post_norm;
    float layer_scalar;
};

struct Rope {
    double theta;
    int hd;
    long len = 0;
    float *cos = nullptr, *sin = nullptr;
};

struct Ctx {
    int h, p, nl, nh, ff, emb;
    float eps;
    std::vector<Layer> layers;
    uint16_t *ple_model, *emb_proj;
    float *ple_norm, *final_norm;
    std::vector<Rope> ropes;
    cublasHandle_t blas = nullptr;
    cudaStream_t stream = nullptr;
    // Work (sized for `cap` rows)
    long cap = 0;
    float *hidden = nullptr, *ple = nullptr, *out = nullptr;
    uint16_t *xb = nullptr, *t = nullptr, *qkv = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *a = nullptr,
             *o = nullptr, *gu = nullptr, *gate = nullptr, *pg = nullptr, *hb = nullptr, *pgb = nullptr;
    int* pos = nullptr;
    std::vector<void*> allocs;
    std::string err;
};

#define CKR(call)                                                                              \
    do {                                                                                       \
        cudaError_t e_ = (call);                                                               \
        if (e_ != cudaSuccess) {                                                               \
            c->err = std::string(#call) + ": " + cudaGetErrorString(e_);                       \
            return -3;                                                                         \
        }                                                                                      \
    } while (0)
#define CKB(call)                                                                              \
    do {                                                                                       \
        cublasStatus_t s_ = (call);                                                            \
        if (s_ != CUBLAS_STATUS_SUCCESS) {                                                     \
            c->err = std::string(#call) + ": cuBLAS status " + std::to_string((int)s_);        \
            return -3;                                                                         \
        }                                                                                      \
    } while (0)

static int dalloc(Ctx* c, void** p, size_t bytes) {
    CKR(cudaMalloc(p, bytes ? bytes : 16));
    c->allocs.push_back(*p);
    return 0;
}
static int upload(Ctx* c, void** dst, const void* src, size_t bytes) {
    if (dalloc(c, dst, bytes)) return -3;
    CKR(cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice));
    return 0;
}

// y[m, n] = x[m, k] . w[n, k]^T, bf16 in, f32 accumulate, y f32 or bf16 (Gpu::gemm_bf16).
static int gemm_bf16(Ctx* c, const uint16_t* x, int m, int k, const uint16_t* w, int n, void* y, bool y_bf16) {
    const float alpha = 1.f, beta = 0.f;
    CKB(cublasGemmEx(c->blas, CUBLAS_OP_T, CUBLAS_OP_N, n, m, k, &alpha, w, CUDA_R_16BF, k, x, CUDA_R_16BF, k, &beta, y,
                     y_bf16 ? CUDA_R_16BF : CUDA_R_32F, n, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT));
    return 0;
}

static int ensure_rope(Ctx* c, long max_len) {
    for (Rope& r : c->ropes) {
        if (r.len >= max_len) continue;
        const long len = ((max_len + 255) / 256) * 256;
        const int half = r.hd / 2;
        std::vector<float> inv(half);
        for (int i = 0; i < half; i++) inv[i] = 1.0f / powf((float)r.theta, (float)(2 * i) / (float)r.hd);
        std::vector<float> cs((size_t)len * r.hd), sn((size_t)len * r.hd);
        for (long t = 0; t < len; t++)
            for (int i = 0; i < half; i++) {
                const float f = (float)t * inv[i];
                const float s = sinf(f), co = cosf(f);
                cs[t * r.hd + i] = cs[t * r.hd + half + i] = co;
                sn[t * r.hd + i] = sn[t * r.hd + half + i] = s;
            }
        if (upload(c, (void**)&r.cos, cs.data(), cs.size() * 4) || upload(c, (void**)&r.sin, sn.data(), sn.size() * 4))
            return -3;
        r.len = len;
    }
    return 0;
}

static int ensure_work(Ctx* c, long rows) {
    if (rows <= c->cap) return 0;
    int q_w = 0, kv_w = 0, qkv_w = 0;
    for (const Layer& L : c->layers) {
        q_w = std::max(q_w, c->nh * L.hd);
        kv_w = std::max(kv_w, L.nkv * L.hd);
        qkv_w = std::max(qkv_w, (c->nh + 2 * L.nkv) * L.hd);
    }
    struct B {
        void** p;
        size_t bytes;
    } bufs[] = {{(void**)&c->hidden, (size_t)rows * c->h * 4},    {(void**)&c->ple, (size_t)rows * c->nl * c->p * 4},
                {(void**)&c->out, (size_t)rows * c->emb * 4},     {(void**)&c->xb, (size_t)rows * c->h * 2},
                {(void**)&c->t, (size_t)rows * c->h * 2},          {(void**)&c->qkv, (size_t)rows * qkv_w * 2},
                {(void**)&c->q, (size_t)rows * q_w * 2},           {(void**)&c->k, (size_t)rows * kv_w * 2},
                {(void**)&c->v, (size_t)rows * kv_w * 2},          {(void**)&c->a, (size_t)rows * q_w * 2},
                {(void**)&c->o, (size_t)rows * c->h * 2},          {(void**)&c->gu, (size_t)rows * 2 * c->ff * 2},
                {(void**)&c->gate, (size_t)rows * c->ff * 2},      {(void**)&c->pg, (size_t)rows * c->p * 2},
                {(void**)&c->hb, (size_t)rows * c->h * 2},         {(void**)&c->pgb, (size_t)rows * c->p * 2},
                {(void**)&c->pos, (size_t)rows * 4}};
    for (B& b : bufs) {
        if (*b.p) {
            cudaFree(*b.p);
            for (auto& a : c->allocs)
                if (a == *b.p) a = nullptr;
        }
        if (dalloc(c, b.p, b.bytes)) return -3;
    }
    c->cap = rows;
    return 0;
}

// GpuText::enqueue for one pass of `lens` (src/gpu/text.rs:350-433), bf16 mode, attention per sequence.
static int enqueue(Ctx* c, const int* lens, int n_seq, long rows) {
    const int h = c->h, p = c->p, nl = c->nl, nh = c->nh, ff = c->ff;
    const float eps = c->eps;
    cudaStream_t s = c->stream;
    // ple = rmsnorm(embeds . W^T * h^-0.5) * ple_norm: the f32 input is rounded to bf16 first
    // (matmul_nt_bf16), the product is f32, then the in-place norm with the pre-scale.
    to_bf16<<<blocks_1d(rows * h, 4 * 256), 256, 0, s>>>(c->hidden, c->xb, rows * h, NEG_INF, POS_INF);
    if (gemm_bf16(c, c->xb, (int)rows, h, c->ple_model, nl * p, c->ple, false)) return -3;
    rms_norm<<<(unsigned)(rows * nl), norm_threads(p), 0, s>>>(nullptr, c->ple, c->ple_norm, (int)(rows * nl), p, eps, 1,
                                                                powf((float)h, -0.5f), NEG_INF, POS_INF, NEG_INF, POS_INF, 0);
    rms_norm_fb<<<(unsigned)rows, norm_threads(h), 0, s>>>(c->hidden, c->t, c->layers[0].input_ln, (int)rows, h, eps, 1, 1.f,
                                                            NEG_INF, POS_INF, NEG_INF, POS_INF, 0);
    for (int i = 0; i < nl; i++) {
        const Layer& L = c->layers[i];
        const int hd = L.hd, nkv = L.nkv, S = nh + 2 * nkv, w = S * hd;
        const Rope* tab = nullptr;
        for (const Rope& r : c->ropes)
            if (r.theta == L.theta && r.hd == hd) tab = &r;
        if (gemm_bf16(c, c->t, (int)rows, h, L.qkv, w, c->qkv, true)) return -3;
        const unsigned qb = (unsigned)((rows * S + 7) / 8);
        if (hd == 256)
            qkv_post_w8r_bb<<<qb, 256, 0, s>>>(c->qkv, c->qkv + nh * hd, c->qkv + (nh + nkv) * hd, w, w, w, c->q, c->k, c->v,
                                               L.q_norm, L.k_norm, tab->cos, tab->sin, c->pos, (int)rows, nh, nkv, hd, hd, eps);
        else
            qkv_post_w16r_bb<<<qb, 256, 0, s>>>(c->qkv, c->qkv + nh * hd, c->qkv + (nh + nkv) * hd, w, w, w, c->q, c->k, c->v,
                                                L.q_norm, L.k_norm, tab->cos, tab->sin, c->pos, (int)rows, nh, nkv, hd, hd, eps);
        long row0 = 0;
        for (int sq = 0; sq < n_seq; sq++) {
            const int n = lens[sq];
            const dim3 grid((unsigned)((n + 63) / 64), (unsigned)nh);
            if (hd == 256)
                flash_attn_d256_bb<<<grid, 128, 0, s>>>(c->q, c->k, c->v, c->a, (int)row0, n, nh, nkv, L.window, 1.f, nh * hd,
                                                        nkv * hd);
            else
                flash_attn_d512_bb<<<grid, 256, FLASH_D512_SMEM, s>>>(c->q, c->k, c->v, c->a, nullptr, (int)row0, n, nh, nkv,
                                                                      L.window, 1.f, nh * hd, nkv * hd);
            row0 += n;
        }
        if (gemm_bf16(c, c->a, (int)rows, nh * hd, L.o, h, c->o, true)) return -3;
        add_norm_bb<<<(unsigned)rows, norm_threads(h), 0, s>>>(c->hidden, c->o, L.post_attn_ln, c->t, L.pre_ff_ln, (int)rows,
                                                                 h, eps, 1.f, NEG_INF, POS_INF, 0, NEG_INF, POS_INF, NEG_INF,
                                                                 POS_INF);
        if (gemm_bf16(c, c->t, (int)rows, h, L.gu, 2 * ff, c->gu, true)) return -3;
        gelu_mul_bb<<<blocks_1d(rows * ff), 256, 0, s>>>(c->gate, c->gu, c->gu + ff, rows * ff, ff, 2 * ff, 2 * ff);
        if (gemm_bf16(c, c->gate, (int)rows, ff, L.down, h, c->o, true)) return -3;
        add_norm_bb<<<(unsigned)rows, norm_threads(h), 0, s>>>(c->hidden, c->o, L.post_ff_ln, c->hb, nullptr, (int)rows, h,
                                                                 eps, 1.f, NEG_INF, POS_INF, 0, NEG_INF, POS_INF, NEG_INF,
                                                                 POS_INF);
        if (gemm_bf16(c, c->hb, (int)rows, h, L.pg, p, c->pg, true)) return -3;
        ple_gate_bb<<<blocks_1d(rows * p), 256, 0, s>>>(c->pgb, c->pg, c->ple, (int)rows, p, nl, i);
        if (gemm_bf16(c, c->pgb, (int)rows, p, L.pp, h, c->o, true)) return -3;
        const float* next_w = (i + 1 < nl) ? c->layers[i + 1].input_ln : c->final_norm;
        add_norm_bb<<<(unsigned)rows, norm_threads(h), 0, s>>>(c->hidden, c->o, L.ple_post_norm, c->t, next_w, (int)rows, h,
                                                                 eps, L.layer_scalar, NEG_INF, POS_INF, 0, NEG_INF, POS_INF,
                                                                 NEG_INF, POS_INF);
    }
    if (gemm_bf16(c, c->t, (int)rows, h, c->emb_proj, c->emb, c->out, false)) return -3;
    CKR(cudaGetLastError());
    return 0;
}

}  // namespace refgpu

using namespace refgpu;

extern "C" {

// Dimensions and per-layer settings: dims = {hidden, ple, layers, heads, ff, emb}; per layer
// hd[l], nkv[l], window[l] (< 0 global), theta[l], layer_scalar[l]. Weight pointers (host): per layer
// 13 pointers in the order qkv, o, gate|up, down, ple_gate, ple_proj (bf16 bits, [out, in]), then
// input_ln, post_attn_ln, pre_ff_ln, post_ff_ln, q_norm, k_norm, ple_post_norm (f32); then globals
// ple_model (bf16), emb_proj (bf16), ple_norm, final_norm (f32).
int refgpu_open(int device, const int* dims, float eps, const int* hd, const int* nkv, const int* window, const double* theta,
                const float* layer_scalar, const void* const* layer_w, const void* const* global_w, void** out) {
    Ctx* c = new Ctx();
    *out = nullptr;
    if (cudaSetDevice(device) != cudaSuccess) {
        delete c;
        return -3;
    }
    c->h = dims[0], c->p = dims[1], c->nl = dims[2], c->nh = dims[3], c->ff = dims[4], c->emb = dims[5];
    c->eps = eps;
    const size_t h = c->h, p = c->p, ff = c->ff, nh = c->nh;
    for (int l = 0; l < c->nl; l++) {
        Layer L{};
        L.hd = hd[l], L.nkv = nkv[l], L.window = window[l], L.theta = theta[l], L.layer_scalar = layer_scalar[l];
        const void* const* w = layer_w + 13 * l;
        const size_t qkv_rows = (nh + 2 * L.nkv) * L.hd;
        int rc = upload(c, (void**)&L.qkv, w[0], qkv_rows * h * 2) | upload(c, (void**)&L.o, w[1], h * nh * L.hd * 2) |
                 upload(c, (void**)&L.gu, w[2], 2 * ff * h * 2) | upload(c, (void**)&L.down, w[3], h * ff * 2) |
                 upload(c, (void**)&L.pg, w[4], p * h * 2) | upload(c, (void**)&L.pp, w[5], h * p * 2) |
                 upload(c, (void**)&L.input_ln, w[6], h * 4) | upload(c, (void**)&L.post_attn_ln, w[7], h * 4) |
                 upload(c, (void**)&L.pre_ff_ln, w[8], h * 4) | upload(c, (void**)&L.post_ff_ln, w[9], h * 4) |
                 upload(c, (void**)&L.q_norm, w[10], L.hd * 4) | upload(c, (void**)&L.k_norm, w[11], L.hd * 4) |
                 upload(c, (void**)&L.ple_post_norm, w[12], h * 4);
        if (rc) {
            fprintf(stderr, "refgpu_open: %s\n", c->err.c_str());
            delete c;
            return -3;
        }
        c->layers.push_back(L);
        bool have = false;
        for (const Rope& r : c->ropes) have |= (r.theta == L.theta && r.hd == L.hd);
        if (!have) {
            Rope r;
            r.theta = L.theta;
            r.hd = L.hd;
            c->ropes.push_back(r);
        }
    }
    int rc = upload(c, (void**)&c->ple_model, global_w[0], (size_t)c->nl * p * h * 2) |
             upload(c, (void**)&c->emb_proj, global_w[1], (size_t)c->emb * h * 2) |
             upload(c, (void**)&c->ple_norm, global_w[2], p * 4) | upload(c, (void**)&c->final_norm, global_w[3], h * 4);
    if (rc || cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cublasCreate(&c->blas) != CUBLAS_STATUS_SUCCESS || cublasSetStream(c->blas, c->stream) != CUBLAS_STATUS_SUCCESS ||
        cublasSetMathMode(c->blas, CUBLAS_TF32_TENSOR_OP_MATH) != CUBLAS_STATUS_SUCCESS ||
        cudaFuncSetAttribute(flash_attn_d512_bb, cudaFuncAttributeMaxDynamicSharedMemorySize, FLASH_D512_SMEM) != cudaSuccess) {
        fprintf(stderr, "refgpu_open: set-up failed %s\n", c->err.c_str());
        delete c;
        return -3;
    }
    *out = c;
    return 0;
}

// One forward_packed pass: host embeds [rows, hidden] in, host per-token states [rows, emb] out
// (H2D, enqueue, D2H as GpuText::forward_packed). *device_ms: CUDA-event time of the enqueued layers.
int refgpu_forward(void* handle, const float* embeds, const int* lens, int n_seq, float* out, float* device_ms) {
    Ctx* c = (Ctx*)handle;
    long rows = 0, max_len = 0;
    for (int i = 0; i < n_seq; i++) {
        if (lens[i] <= 0) return -1;
        rows += lens[i];
        max_len = std::max<long>(max_len, lens[i]);
    }
    if (ensure_work(c, rows) || ensure_rope(c, max_len)) return -3;
    std::vector<int> pos(rows);
    for (long r = 0, s = 0; s < n_seq; s++)
        for (int i = 0; i < lens[s]; i++) pos[r++] = i;
    cudaEvent_t e0, e1;
    CKR(cudaEventCreate(&e0));
    CKR(cudaEventCreate(&e1));
    CKR(cudaMemcpyAsync(c->hidden, embeds, rows * c->h * 4, cudaMemcpyHostToDevice, c->stream));
    CKR(cudaMemcpyAsync(c->pos, pos.data(), rows * 4, cudaMemcpyHostToDevice, c->stream));
    CKR(cudaEventRecord(e0, c->stream));
    if (enqueue(c, lens, n_seq, rows)) return -3;
    CKR(cudaEventRecord(e1, c->stream));
    CKR(cudaMemcpyAsync(out, c->out, rows * c->emb * 4, cudaMemcpyDeviceToHost, c->stream));
    CKR(cudaStreamSynchronize(c->stream));
    float ms = 0.f;
    CKR(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (device_ms) *device_ms = ms;
    return 0;
}

const char* refgpu_error(void* handle) { return handle ? ((Ctx*)handle)->err.c_str() : ""; }

void refgpu_close(void* handle) {
    Ctx* c = (Ctx*)handle;
    if (!c) return;
    if (c->stream) cudaStreamSynchronize(c->stream);
    for (void* p : c->allocs)
        if (p) cudaFree(p);
    if (c->blas) cublasDestroy(c->blas);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

}  // extern "C"

// Internal host-side interface of the kernels (not part of the C ABI; see include/eg2.h for that).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace eg2 {

typedef uint16_t bf16_t;

enum GemmKind : int { GEMM_BF16 = 0, GEMM_TF32 = 1, GEMM_F32 = 2 };

enum EpiMode : int {
    EPI_STORE = 0,     // out = acc * scale (bf16 or f32)
    EPI_GELU_GU = 1,   // weights interleaved in 128-row gate / up halves per 256-row block: out = gelu(g) * u
    EPI_PLE_GATE = 2,  // out = gelu(acc) * aux[row * aux_ld + aux_off + col]
    EPI_QKV = 3,       // fused projection [q | k | v] -> per-head RMSNorm (+ weights on q, k) and RoPE on
                       // q, k, written to q [M, nh, hd], k / v [M, nkv, hd]; needs 256 % hd == 0
    EPI_ADD_NORM = 4,  // N = 512, bf16 inputs: residual update and norms of add_norm() on the accumulator
                       // (see AddNormEpilogue); `out` receives t (bf16, ldo), the accumulator is not stored
    EPI_GROUP_NORM = 5,  // N = 512 g, bf16 inputs: each 512-column group of acc * scale is RMS-normalised
                         // (an.eps) and multiplied by an.w1[col % 512]; `out` f32 [M, ldo]
    EPI_QKV_PAIR = 6,    // EPI_QKV for head_dim 512 (RoPE over the whole head): one 512-column group per
                         // head, the two 256-column halves on a 2-CTA cluster. The weight rows of each head
                         // must be in the pair layout (qkv_pair_row): half r holds head channels
                         // [128 r, 128 r + 128) and [256 + 128 r, 256 + 128 r + 128), so every rotated pair
                         // (i, i + 256) is inside one half
    EPI_PLE_FUSED = 7,   // the PLE gate with this layer's PLE slice computed in the same kernel: two products per
                         // tile, g = A . W^T and p = A2 . W2[aux_off .., :]^T (A2, W2: tensor maps of the
                         // launch), out = bf16(gelu(g) * (p * scale / rms(p * scale) * an.w1[col])), the RMS over
                         // each row's 512 columns; clusters of four CTAs, one per 128-column quarter
};

// Pair layout of a 512-channel head: weight row n' (0..511) of the permuted head holds original
// channel qkv_pair_row(n').
inline int qkv_pair_row(int np) {
    const int r = (np >> 7) & 1, hi = np >> 8;  // [0,128) -> 0, [128,256) -> 256, [256,384) -> 128, [384,512) -> 384
    return (np & 127) + 128 * hi + 256 * r;
}

// EPI_ADD_NORM, with o the GEMM result row (512 wide):
//   h = (h + o / rms(o) * w1) * scalar;  out = w2 ? h / rms(h) * w2 : h   (rms(x) = sqrt(mean(x^2) + eps))
// Runs as clusters of two CTAs, one per 256-column half of a 128-row block; the two halves of each
// row's sum of squares are exchanged through distributed shared memory.
struct AddNormEpilogue {
    float* h = nullptr;          // [M, 512] f32 residual stream, updated in place
    const float* w1 = nullptr;   // [512]
    const float* w2 = nullptr;   // [512] or nullptr
    float eps = 1e-6f;
    float scalar = 1.f;
};

struct QkvEpilogue {
    void *q = nullptr, *k = nullptr, *v = nullptr;
    const float *wq = nullptr, *wk = nullptr;
    const float* inv_freq = nullptr;  // part / 2 RoPE inverse frequencies (f32, as the reference computes them)
    const int* pos = nullptr;         // position of row r, rotation part pi: pos[r * pos_stride + pi] (nullptr: r)
    int pos_stride = 1;
    int nh = 0, nkv = 0, hd = 0, part = 0;     // part: rotation width (hd, or hd / 2 for 2-D RoPE)
    float eps = 1e-6f;
};

struct GemmEpilogue {
    int mode = EPI_STORE;
    int out_f32 = 0;          // EPI_STORE with bf16 inputs: write f32 instead of bf16
    void* out = nullptr;      // [M, ldo] (EPI_GELU_GU: N/2 valid columns)
    long ldo = 0;
    const float* aux = nullptr;
    long aux_ld = 0;
    int aux_off = 0;
    float scale = 1.f;
    // EPI_STORE, CTA pairs: split the K range into ksplit equal slices, slice s of every tile written
    // (f32) at out + s * split_stride -- for passes too short to spread the weights over the SMs.
    int ksplit = 1;
    long split_stride = 0;
    QkvEpilogue qkv;
    AddNormEpilogue an;
};

// Number of SMs of the current device (cached per device).
int num_sms();
// Launch the tensor-core kernels as programmatic dependents of the previous kernel on the stream
// (their prologue overlaps its tail); EG2_NO_PDL=1 turns it off.
bool pdl_enabled();

// 2-D K-major tensor map with 128-byte swizzle: `inner` elements per row (the K extent),
// `outer` rows, `row_bytes` between rows; box = box_inner x box_outer.
int make_tmap_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                 uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);
// 3-D variant: dims (d0, d1, d2) with byte strides s1 (dim 1) and s2 (dim 2); box (b0, b1, b2).
int make_tmap_3d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                 uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2,
                 CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

// Whether EPI_QKV applies to a head configuration (whole heads per 256-column tile).
bool qkv_fusable(const QkvEpilogue& q);
bool qkv_pair_fusable(const QkvEpilogue& q);
// C = A . W^T on tcgen05 (bf16 or tf32 inputs). N must be a multiple of 256, K of 64 (bf16) / 32 (tf32).
int gemm_tc(GemmKind kind, const void* A, long lda, const void* W, long ldw, int M, int N, int K,
            const GemmEpilogue& epi, cudaStream_t s);
// EPI_PLE_FUSED (bf16, N = K = 512): out[M, 512] = bf16(gelu(t . w_gate^T) * plenorm(x . w_ple[layer]^T)),
// where plenorm(v) = rms_norm(v * scale) * norm_w over the row's 512 columns (the PLE prologue of
// src/text.rs:145-149 for one layer, fused into that layer's gate, src/text.rs:218-224). w_ple_all is the
// stacked [layers * 512, 512] PLE model projection.
int gemm_ple_fused(const bf16_t* t, const bf16_t* x, const bf16_t* w_gate, const bf16_t* w_ple_all, int layer,
                   const float* norm_w, float scale, float eps, bf16_t* out, int M, cudaStream_t s);
// f32 CUDA-core GEMM (the float32 precision path): out f32 [M, ldo] = scale * A . W^T.
int gemm_f32(const float* A, long lda, const float* W, long ldw, float* out, long ldo, int M, int N, int K, float scale,
             cudaStream_t s);

// ---- row kernels (rowops.cu) ----
template <typename TO>
int rms_norm_rows(const float* x, TO* out, const float* w, long rows, int dim, float eps, float pre, cudaStream_t s);
int rms_norm_inplace(float* x, const float* w, long rows, int dim, float eps, float pre, cudaStream_t s);
// h = (h + rmsnorm(o) * w1) * scalar; then optionally t = rmsnorm(h) * w2 (w2 == nullptr: t = h copy).
template <typename TI, typename TT>
int add_norm(float* h, const TI* o, const float* w1, TT* t, const float* w2, long rows, int dim, float eps,
             float scalar, cudaStream_t s);
// GELU(g) x ple[:, layer] (out [rows, p]) for g given as nsplit f32 partial sums stride apart.
template <typename TO>  // bf16_t (bf16 contexts) or float (TF32)
int ple_gate_split(const float* part, int nsplit, long stride, const float* ple, long ple_ld, int ple_off, TO* out,
                   long rows, int p, cudaStream_t s);
// K-split partial sums (f32, stride apart, added in slice order) of the gate|up projection -> gelu(gate) * up,
// and of the q|k|v projection -> qkv_post (TF32 passes of few rows).
int gelu_gu_split(const float* part, int nsplit, long stride, float* out, long rows, int ff, cudaStream_t s);
int qkv_post_split(const float* qkv, int nsplit, long split_stride, float* q, float* k, float* v, const float* wq,
                   const float* wk, const float* cs, const float* sn, int rope_w, const int* pos, long rows, int nh,
                   int nkv, int hd, int part, float eps, cudaStream_t s);
// add_norm over o given as nsplit f32 partial sums o_stride elements apart (dim 512; t bf16 or f32).
template <typename TT>
int add_norm_split(float* h, const float* o, int nsplit, long o_stride, const float* w1, TT* t, const float* w2,
                   long rows, int dim, float eps, float scalar, cudaStream_t s);
// Per-head RMSNorm (q, k weighted; v not) and RoPE on q and k, from the fused projection output
// qkv[row, (nh + 2 nkv) * hd]. cs/sn: [positions, rope_w] tables; part = rotation width (hd or hd / 2).
template <typename TI, typename TO>
int qkv_post(const TI* qkv, TO* q, TO* k, TO* v, const float* wq, const float* wk, const float* cs, const float* sn,
             int rope_w, const int* pos, long rows, int nh, int nkv, int hd, int part, float eps, cudaStream_t s);
template <typename TI, typename TO>
int gelu_gu(const TI* gu, TO* out, long rows, int ff, cudaStream_t s);
template <typename TI, typename TO>
int ple_gate(const TI* g, TO* out, const float* ple, long rows, int p, int n_layers, int layer, cudaStream_t s);
// dims_dev: device array of n_dims cut widths (the first is normally dim itself); out row stride out_stride.
// scratch: pool_scratch_doubles(n_seq, max_len, dim) doubles of partial sums.
int pool_scratch_doubles(int n_seq, int max_len, int dim);
int pool_rows(const float* x, const int* seq_start, const int* seq_len, int n_seq, int max_len, int dim,
              const int* dims_dev, int n_dims, int out_stride, float* out, double* scratch, cudaStream_t s);
// pos / seq_start / seq_len of every row of a pass from its n_seq + 1 sequence offsets (device memory).
int row_meta(const int* off, int n_seq, long rows, int* pos, int* st, int* ln, cudaStream_t s);
// embed_gather, the bf16 copy of its result and the first pre-norm in one kernel (h = 512).
int embed_gather_norm(const bf16_t* table, long vocab, int h, const uint32_t* ids, long n, float scale, float* hidden,
                      bf16_t* xb, bf16_t* t, const float* w, float eps, int* bad, cudaStream_t s);
int embed_gather(const bf16_t* table, long vocab, int h, const uint32_t* ids, long n, float scale, float* out,
                 int* bad, cudaStream_t s);
template <typename TO>
int cast_rows(const float* x, TO* out, long n, float mul, float add, cudaStream_t s);
int widen_bf16(const bf16_t* x, float* out, long n, cudaStream_t s);
int vision_add_positions(float* h, const float* table, const int* pos, long n, int hdim, int pe, cudaStream_t s);
int vision_pool(const float* x, float* out, int gh, int gw, int hdim, int k, float root, cudaStream_t s);

// ---- attention ----
// Tile list for the tensor-core kernel: one entry per (sequence, query tile): {row0, len, q0}.
struct AttnTile {
    int row0, len, q0;
};
// Tensor-core flash attention, bf16 q/k/v/out, GQA-packed query tiles (attention_tc.cu). A tile is
// (row0, len, q0): query tokens q0.. of the len rows from row0, keys among those rows. With
// seq_start / seq_len (per row: first row and length of its sequence) each row also masks the keys
// outside its own sequence, so one tile may hold several whole short sequences (q0 = 0); without them
// a tile's rows are one sequence.
int attention_tc(const bf16_t* q, const bf16_t* k, const bf16_t* v, bf16_t* out, long rows, const AttnTile* tiles,
                 int n_tiles, int nh, int nkv, int hd, int window, cudaStream_t s, const int* seq_start = nullptr,
                 const int* seq_len = nullptr);
// attention_tc with its tile list built in a fixed device array instead of allocated memory (noalloc.cu).
int attention_noalloc(const bf16_t* q, const bf16_t* k, const bf16_t* v, bf16_t* out, const int32_t* lens, int n_seq,
                      int nh, int nkv, int hd, int window, cudaStream_t s);
// Query tokens per tile of attention_tc for a head configuration.
int attention_tc_tile_tokens(int nh, int nkv, int hd);
// Failure-detection probe: a bounded wait on a barrier nothing arrives on (probe.cu).
int wait_timeout_probe(unsigned long long limit_ns, cudaStream_t s);
// CUDA-core attention (f32 arithmetic; bf16 or f32 storage), one warp per (row, head).
template <typename T>
int attention_simt(const T* q, const T* k, const T* v, T* out, const int* seq_start, const int* seq_len, long rows,
                   int nh, int nkv, int hd, int window, cudaStream_t s);

}  // namespace eg2

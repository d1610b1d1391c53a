/*
 * eg2.h -- C ABI of the B200-native EmbeddingGemma 2 text-backbone and vision-tower library
 * (libeg2_b200.so, built for sm_100a).
 *
 * It is the drop-in for the reference engine's device backends. Each entry point names the
 * reference interface it replaces (paths inside the reference project):
 *
 *   eg2_open / eg2_close          GpuText::from_cpu + Gpu::new (src/gpu/text.rs:177-219,
 *                                 src/gpu/mod.rs:281-403), reading the checkpoint like
 *                                 Weights::open + TextModel::load (src/weights.rs:46-86, src/text.rs:67-114)
 *   eg2_embed_tokens              TextBackend::embed_tokens (src/backend.rs:64-70, src/text.rs:53-64)
 *   eg2_forward_packed            TextBackend::forward_packed (src/backend.rs:73-79,
 *                                 src/gpu/text.rs:436-529): [rows, 512] f32 in, [rows, 768] f32 out
 *   eg2_embed_packed              EmbeddingGemma2::embed_prepared's text tail + truncate_and_normalize
 *                                 (src/model.rs:508-540, :677-688): ids in, pooled L2-normalised
 *                                 embeddings (and Matryoshka cuts) out, all on the device
 *   eg2_vision_encode             VisionBackend::encode (src/backend.rs:88-95, src/gpu/vision.rs:97-219)
 *   eg2_gemm                      Gpu::gemm_bf16 / Gpu::matmul_nt (src/gpu/mod.rs:554-630)
 *   eg2_attention                 Gpu::attention_act / attention_flash_packed (src/gpu/mod.rs:1217-1599)
 *
 * Conventions: every function returns 0 on success or a negative EG2_ERR_* code; the message of
 * the last failure is available from eg2_last_error. A failure before the result is written
 * leaves the output untouched. Calls on one context are serialised internally (the reference
 * holds one lock per device, src/gpu/mod.rs:472-475); different contexts (GPUs) may be driven
 * concurrently from different host threads. Host pointers are plain host memory; "_device"
 * variants take device pointers and an optional CUDA stream (NULL: the context's own stream).
 */
#ifndef EG2_H
#define EG2_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct eg2_ctx eg2_ctx;

/* Precision of the matrix products (src/backend.rs:17-27). */
enum {
    EG2_F32 = 0,  /* f32 CUDA-core GEMMs and attention: float32 profile */
    EG2_TF32 = 1, /* TF32 tensor-core GEMMs, f32 activations: tf32 profile */
    EG2_BF16 = 2  /* bf16 tensor-core GEMMs and attention, f32 residual / norms: bf16 profile */
};

enum {
    EG2_OK = 0,
    EG2_ERR_INVALID = -1, /* bad argument (sizes, ids out of range, empty sequence) */
    EG2_ERR_OOM = -2,     /* device or pinned host memory exhausted */
    EG2_ERR_CUDA = -3,    /* a CUDA call failed */
    EG2_ERR_TIMEOUT = -4, /* a bounded device wait ran out (the kernel returned an error status) */
    EG2_ERR_IO = -5       /* checkpoint or config unreadable / malformed */
};

/* Open `model_dir` (config.json + model.safetensors in the reference's layout) on CUDA device
 * `device`. Loads the text tower; the vision tower is loaded when present. */
int eg2_open(int device, int precision, const char* model_dir, eg2_ctx** out);
void eg2_close(eg2_ctx* ctx);
/* Message of the last failure on `ctx` (or of the last failed eg2_open when ctx is NULL). */
const char* eg2_last_error(const eg2_ctx* ctx);

/* Model dimensions: hidden size, output (embedding) width, vocabulary size, layers. */
int eg2_text_dims(const eg2_ctx* ctx, int* hidden, int* embedding_dim, int64_t* vocab, int* layers);

/* Scaled token embeddings embed_tokens[id] * sqrt(hidden) for `n` ids into out [n, hidden]. */
int eg2_embed_tokens(eg2_ctx* ctx, const uint32_t* ids, int64_t n, float* out);

/* Per-token states [rows, embedding_dim] for `n_seq` sequences packed back to back
 * (rows = sum(lens)); embeds [rows, hidden]. Host buffers. */
int eg2_forward_packed(eg2_ctx* ctx, const float* embeds, const int32_t* lens, int n_seq, float* out);
/* Same with device buffers; `lens` stays a host array. Work is enqueued on `stream` (or the
 * context's stream) and the call returns after it completes. A call of several passes (see
 * eg2_plan_passes) writes each pass's rows once that pass has completed: an argument error leaves
 * `out` untouched, a device failure in a later pass leaves the earlier passes' rows written. */
int eg2_forward_packed_device(eg2_ctx* ctx, const float* embeds, const int32_t* lens, int n_seq, float* out,
                              void* stream);

/* Token ids of `n_seq` sequences packed back to back -> per sequence, the L2-normalised mean of
 * the per-token states, followed by its Matryoshka cuts: for each dims[i] (dims[0] is normally
 * embedding_dim) the first dims[i] components re-normalised. out [n_seq, sum(dims)]. Host buffers. */
int eg2_embed_packed(eg2_ctx* ctx, const uint32_t* ids, const int32_t* lens, int n_seq, const int32_t* dims,
                     int n_dims, float* out);
int eg2_embed_packed_device(eg2_ctx* ctx, const uint32_t* ids, const int32_t* lens, int n_seq, const int32_t* dims,
                            int n_dims, float* out, void* stream);

/* Pass policy of eg2_forward_packed / eg2_embed_packed (both variants). A call is split into device
 * passes of consecutive sequences in call order, each of at most max_rows packed rows (a longer
 * sequence gets a pass of its own), as the reference's embed_prepared packs inputs into passes of at
 * most PACK_TOKENS rows (src/model.rs:157-158, :508-521), so any call runs in a bounded workspace;
 * in bf16 contexts the sequences of at most precise_max tokens form their own passes, computed in
 * TF32 (their bf16 rounding errors are not averaged out by the mean pool). Each pass gives the same
 * bits as a call holding only its sequences. eg2_plan_passes computes the plan without a device:
 * pass_of_seq[n_seq] receives each sequence's pass, pass_precise (room for n_seq entries, may be NULL)
 * 1 for the TF32 passes; it returns the number of passes or a negative EG2_ERR_* code.
 * eg2_pass_policy reports a context's max_rows and precise_max (0 when no pass runs in TF32). */
int eg2_plan_passes(const int32_t* lens, int n_seq, int64_t max_rows, int precise_max, int32_t* pass_of_seq,
                    int32_t* pass_precise);
int eg2_pass_policy(const eg2_ctx* ctx, int64_t* max_rows, int* precise_max);

/* Vision tower over one patched image: patches [n, 3*p*p] in [0, 1], pos_xy [n, 2] (x, y),
 * n = grid_h * grid_w. out_pooled [n/k^2, vision_hidden] (3x3-pooled states * sqrt(hidden), the
 * reference GPU tower's output) and out_soft [n/k^2, text_hidden] (after the multimodal
 * embedder); either may be NULL. */
int eg2_vision_encode(eg2_ctx* ctx, const float* patches, const int32_t* pos_xy, int grid_h, int grid_w,
                      float* out_pooled, float* out_soft);

/* The vision tower over n_images images of one patch grid, in one device pass (the reference encodes
 * image by image, VisionBackend::encode, src/gpu/vision.rs:97-219; here the images are stacked so
 * the GEMMs and the attention grid cover all of them). patches [n_images, n, 3*p*p]; pos_xy [n, 2],
 * shared by every image; out_pooled [n_images * n/k^2, vision_hidden], out_soft
 * [n_images * n/k^2, text_hidden], image after image; either may be NULL. Each image's results equal
 * an eg2_vision_encode call on it alone, up to the summation order of the row blocks. */
int eg2_vision_encode_batch(eg2_ctx* ctx, const float* patches, const int32_t* pos_xy, int n_images, int grid_h,
                            int grid_w, float* out_pooled, float* out_soft);

/* Run on a caller-owned CUDA stream (cudaStream_t); NULL restores the context's own stream. */
int eg2_set_stream(eg2_ctx* ctx, void* stream);

/* Per-op device timing (CUDA events around each launch group, like the reference's
 * EGEMMA2_PROFILE marks, src/gpu/mod.rs:437-469). eg2_profile_read writes a JSON object
 * {"label": [ms_total, count], ...} accumulated since enabling. */
int eg2_profile(eg2_ctx* ctx, int enable);
int eg2_profile_read(eg2_ctx* ctx, char* buf, int cap);

/* ---- single ops on device pointers (GEMM sweep and attention checks) ---- */

/* C[M, N] = A[M, K] . W[N, K]^T. kind: EG2_BF16 (bf16 A/W, tcgen05), EG2_TF32 (f32 A/W,
 * tcgen05 TF32), EG2_F32 (f32 CUDA cores). C is f32 when out_f32 != 0 or kind != EG2_BF16,
 * else bf16. N must be a multiple of 256 and K of 64 on the tensor-core kinds. */
int eg2_gemm(int kind, const void* A, int64_t lda, const void* W, int64_t ldw, void* C, int64_t ldc, int M, int N,
             int K, int out_f32, void* stream);

/* Block-diagonal bidirectional attention, scale 1, window radius `window` (< 0: global).
 * q [rows, nh, hd], k / v [rows, nkv, hd], out [rows, nh, hd]; lens host array.
 * kind: EG2_BF16 (bf16 storage, tcgen05 flash kernels: hd 256 or 512 with nh / nkv dividing 128,
 * as in the text layers, or hd 64 with nh == nkv, as in the vision tower; one sequence per query
 * tile), EG2_F32 (f32 CUDA cores, any hd up to 512). */
int eg2_attention(int kind, const void* q, const void* k, const void* v, void* out, const int32_t* lens, int n_seq,
                  int nh, int nkv, int hd, int window, void* stream);

/* No counterpart in the reference. The tensor-core attention of eg2_attention (kind EG2_BF16,
 * same arguments and results) without any device allocation, for callers that cannot call
 * cudaMalloc: engines that hand all device memory to their own pool up front (an allocation behind
 * the pool's back can fail or fragment it), and latency-critical paths that cannot take
 * cudaMalloc's implicit device synchronisation. Its scratch (sequence lengths and the query-tile
 * list) lives in one fixed 1 MiB device array per GPU, held until the process exits; calls with
 * more than 65536 sequences or 65536 query tiles (4 M to 16 M rows: a tile holds 64, 128 or 256
 * query tokens by head layout) return EG2_ERR_INVALID before anything is copied or launched. The
 * first call on a device looks the array's device address up (make that first call before any
 * stream capture). All calls share the
 * array and it keeps the last call's contents: calls that overlap on the GPU (unordered streams or
 * threads) race. The call is asynchronous on `stream`: `lens` in pageable host memory is read before
 * the call returns; in page-locked memory it is read when the stream reaches the copy and must stay
 * unchanged until then. A bounded device wait that ran out is not returned as EG2_ERR_TIMEOUT here:
 * synchronise the stream, then read eg2_device_status() (non-zero: the result is not valid). */
int eg2_attention_noalloc(const void* q, const void* k, const void* v, void* out, const int32_t* lens, int n_seq,
                          int nh, int nkv, int hd, int window, void* stream);

/* Number of kernel launches this library has issued in the process (all contexts). */
long long eg2_launch_count(void);

/* First error code recorded by a device-side bounded wait since the last reset (0: none). */
int eg2_device_status(void);
void eg2_device_status_reset(void);

/* Failure-detection probe. No counterpart in the reference (its kernels have no bounded waits):
 * launches one CTA on `device` that waits on an mbarrier nothing arrives on, bounded by `limit_us`
 * (1 .. 2,000,000) microseconds of wall time -- the same bounded wait every pipeline barrier of the
 * library uses. The wait runs out and records status 4 in the device status word; the call
 * synchronises, stores that status in *device_status, clears it and returns EG2_OK when the context
 * is still usable. Every other entry point reports such a recorded status as EG2_ERR_TIMEOUT. */
int eg2_wait_timeout_probe(int device, unsigned int limit_us, int* device_status);

#ifdef __cplusplus
}
#endif

#endif /* EG2_H */

// Host runtime of the library: checkpoint loading, device weights, per-pass workspace, the text
// backbone and vision tower launch sequences, and the C ABI of include/eg2.h.
//
// Reference counterparts (paths inside the reference project):
//   context + weights upload   Gpu::new, GpuText::from_cpu (src/gpu/mod.rs:281-403, src/gpu/text.rs:177-219)
//   layer launch sequence      GpuText::enqueue (src/gpu/text.rs:350-433)
//   forward_packed             GpuText::forward_packed (src/gpu/text.rs:436-529)
//   RoPE tables                GpuText::ensure_rope (src/gpu/text.rs:227-242), src/ops.rs:293-314
//   vision                     GpuVision::encode (src/gpu/vision.rs:97-219), VisionHead (src/vision.rs:47-170)
//   safetensors                Weights::open (src/weights.rs:46-86)
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/eg2.h"
#include "json.h"
#include "kernels.h"

namespace eg2 {

// ---------------------------------------------------------------------------------------------
// Driver helpers
// ---------------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    });
    return fn;
}

int make_tmap_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                 uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return -3;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -1;
}

int make_tmap_3d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                 uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2, CUtensorMapSwizzle swizzle) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return -3;
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {s1, s2};
    cuuint32_t box[3] = {b0, b1, b2};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = fn(m, dt, 3, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -1;
}

bool pdl_enabled() {
    static const bool on = [] {
        const char* e = getenv("EG2_NO_PDL");
        return !(e && e[0] == '1');
    }();
    return on;
}

int num_sms() {
    static int cache[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
}

// ---------------------------------------------------------------------------------------------
// Errors
// ---------------------------------------------------------------------------------------------
struct Fail {
    int code;
    std::string msg;
};
[[noreturn]] static void fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    throw Fail{code, buf};
}
// On failure the runtime's last-error slot is cleared too, so a later launch check on this thread does
// not report this call's (non-sticky) error as its own.
#define CK(call)                                                                                      \
    do {                                                                                              \
        cudaError_t e_ = (call);                                                                      \
        if (e_ != cudaSuccess) {                                                                      \
            cudaGetLastError();                                                                       \
            fail(e_ == cudaErrorMemoryAllocation ? EG2_ERR_OOM : EG2_ERR_CUDA, "%s: %s (%s:%d)", #call, \
                 cudaGetErrorString(e_), __FILE__, __LINE__);                                         \
        }                                                                                             \
    } while (0)
// Kernel launches issued by this library (all contexts), for the benchmark's launch count.
static std::atomic<long long> g_launches{0};
#define KL(call, what)                                                                         \
    do {                                                                                       \
        int r_ = (call);                                                                       \
        if (r_ != 0) fail(r_ == -1 ? EG2_ERR_INVALID : EG2_ERR_CUDA, "launch of %s failed", what); \
        g_launches.fetch_add(1, std::memory_order_relaxed);                                    \
    } while (0)

// ---------------------------------------------------------------------------------------------
// Safetensors (mmap, BF16 / F16 / F32), checks as src/weights.rs:46-86
// ---------------------------------------------------------------------------------------------
struct TensorInfo {
    std::string dtype;
    std::vector<long> shape;
    size_t start = 0, end = 0;
    long numel() const {
        long n = 1;
        for (long d : shape) n *= d;
        return n;
    }
};

struct SafeTensors {
    void* map = nullptr;
    size_t size = 0;
    size_t data_start = 0;
    std::map<std::string, TensorInfo> index;

    explicit SafeTensors(const std::string& path) {
        int fd = ::open(path.c_str(), O_RDONLY);
        if (fd < 0) fail(EG2_ERR_IO, "opening %s", path.c_str());
        struct stat st;
        fstat(fd, &st);
        size = (size_t)st.st_size;
        map = size ? mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0) : MAP_FAILED;
        ::close(fd);
        if (map == MAP_FAILED) fail(EG2_ERR_IO, "mapping %s", path.c_str());
        if (size < 8) fail(EG2_ERR_IO, "safetensors file too small");
        uint64_t hlen;
        memcpy(&hlen, map, 8);
        if (hlen > size - 8) fail(EG2_ERR_IO, "corrupt safetensors header length in %s", path.c_str());
        data_start = 8 + hlen;
        Json h;
        try {
            h = Json::parse((const char*)map + 8, hlen);
        } catch (std::exception& e) {
            fail(EG2_ERR_IO, "parsing the header of %s: %s", path.c_str(), e.what());
        }
        for (auto& kv : h.obj) {
            if (kv.first == "__metadata__") continue;
            TensorInfo t;
            t.dtype = kv.second.at("dtype").string();
            for (auto& d : kv.second.at("shape").arr) t.shape.push_back(d.integer());
            const auto& off = kv.second.at("data_offsets").arr;
            t.start = (size_t)off.at(0).integer();
            t.end = (size_t)off.at(1).integer();
            long esz = t.dtype == "F32" ? 4 : (t.dtype == "BF16" || t.dtype == "F16") ? 2 : 0;
            if (!esz) fail(EG2_ERR_IO, "tensor %s: unsupported dtype %s", kv.first.c_str(), t.dtype.c_str());
            if (t.end < t.start || data_start + t.end > size || (size_t)(t.numel() * esz) != t.end - t.start)
                fail(EG2_ERR_IO, "tensor %s: bad offsets", kv.first.c_str());
            index[kv.first] = t;
        }
    }
    ~SafeTensors() {
        if (map && map != MAP_FAILED) munmap(map, size);
    }
    bool has(const std::string& n) const { return index.count(n) > 0; }
    const TensorInfo& info(const std::string& n, std::initializer_list<long> shape) const {
        auto it = index.find(n);
        if (it == index.end()) fail(EG2_ERR_IO, "missing tensor `%s`", n.c_str());
        std::vector<long> want(shape);
        if (!want.empty() && it->second.shape != want) {
            // Accept a scalar stored as [] or [1].
            if (!(want.size() == 1 && want[0] == 1 && it->second.numel() == 1))
                fail(EG2_ERR_IO, "tensor `%s` has an unexpected shape", n.c_str());
        }
        return it->second;
    }
    const uint8_t* bytes(const TensorInfo& t) const { return (const uint8_t*)map + data_start + t.start; }
    // Whole tensor as host f32 (BF16 widened exactly as bf16_to_f32, src/weights.rs:189-191).
    std::vector<float> f32(const std::string& n, std::initializer_list<long> shape) const {
        const TensorInfo& t = info(n, shape);
        std::vector<float> out(t.numel());
        const uint8_t* b = bytes(t);
        if (t.dtype == "F32") {
            memcpy(out.data(), b, out.size() * 4);
        } else if (t.dtype == "BF16") {
            for (size_t i = 0; i < out.size(); i++) {
                uint32_t u = (uint32_t)(b[2 * i] | (b[2 * i + 1] << 8)) << 16;
                memcpy(&out[i], &u, 4);
            }
        } else {
            fail(EG2_ERR_IO, "tensor %s: F16 not supported here", n.c_str());
        }
        return out;
    }
};

static uint16_t f32_to_bf16_host(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// ---------------------------------------------------------------------------------------------
// Configuration (src/config.rs:21-66)
// ---------------------------------------------------------------------------------------------
struct TextCfg {
    long vocab = 0;
    int hidden = 0, inter = 0, layers = 0, nh = 0, ple = 0, emb = 0, window = 0;
    float eps = 1e-6f;
    std::vector<int> hd, nkv, sliding;
    std::vector<double> theta;
};
struct VisionCfg {
    bool present = false;
    int hidden = 0, inter = 0, layers = 0, nh = 0, nkv = 0, hd = 0, patch = 0, pool = 0, pos_size = 0;
    float eps = 1e-6f;
    double theta = 100.0;
};

static std::string read_file(const std::string& path) {
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) fail(EG2_ERR_IO, "reading %s", path.c_str());
    std::string s;
    char buf[65536];
    size_t n;
    while ((n = fread(buf, 1, sizeof buf, f)) > 0) s.append(buf, n);
    fclose(f);
    return s;
}

static void parse_config(const std::string& dir, TextCfg& tc, VisionCfg& vc) {
    std::string raw = read_file(dir + "/config.json");
    Json j;
    try {
        j = Json::parse(raw.data(), raw.size());
        const Json& t = j.at("text_config");
        if (t.has("attention_bias") && t.at("attention_bias").kind == Json::Bool && t.at("attention_bias").b)
            fail(EG2_ERR_IO, "attention_bias=true is not supported");
        tc.vocab = t.at("vocab_size").integer();
        tc.hidden = (int)t.at("hidden_size").integer();
        tc.inter = (int)t.at("intermediate_size").integer();
        tc.layers = (int)t.at("num_hidden_layers").integer();
        tc.nh = (int)t.at("num_attention_heads").integer();
        tc.ple = (int)t.at("hidden_size_per_layer_input").integer();
        tc.emb = (int)t.at("embedding_dim").integer();
        tc.window = (int)t.at("sliding_window").integer();
        tc.eps = (float)t.at("rms_norm_eps").number();
        const int hd0 = (int)t.at("head_dim").integer(), nkv0 = (int)t.at("num_key_value_heads").integer();
        const Json& lt = t.at("layer_types");
        const Json& rp = t.at("rope_parameters");
        for (int i = 0; i < tc.layers; i++) {
            const bool sl = lt.arr.at(i).string() == "sliding_attention";
            int hd = hd0, nkv = nkv0;
            if (t.has("per_layer_config")) {
                char k2[16], k1[16];
                snprintf(k2, sizeof k2, "%02d", i);
                snprintf(k1, sizeof k1, "%d", i);
                const Json& plc = t.at("per_layer_config");
                const Json* ov = plc.has(k2) ? &plc.at(k2) : plc.has(k1) ? &plc.at(k1) : nullptr;
                if (ov) {
                    if (ov->has("head_dim") && ov->at("head_dim").kind == Json::Num) hd = (int)ov->at("head_dim").integer();
                    if (ov->has("num_key_value_heads") && ov->at("num_key_value_heads").kind == Json::Num)
                        nkv = (int)ov->at("num_key_value_heads").integer();
                }
            }
            tc.hd.push_back(hd);
            tc.nkv.push_back(nkv);
            tc.sliding.push_back(sl ? 1 : 0);
            tc.theta.push_back(rp.at(sl ? "sliding_attention" : "full_attention").at("rope_theta").number());
        }
        if (j.has("vision_config") && j.at("vision_config").kind == Json::Obj) {
            const Json& v = j.at("vision_config");
            vc.present = true;
            vc.hidden = (int)v.at("hidden_size").integer();
            vc.inter = (int)v.at("intermediate_size").integer();
            vc.layers = (int)v.at("num_hidden_layers").integer();
            vc.nh = (int)v.at("num_attention_heads").integer();
            vc.nkv = (int)v.at("num_key_value_heads").integer();
            vc.hd = (int)v.at("head_dim").integer();
            vc.patch = (int)v.at("patch_size").integer();
            vc.pool = (int)v.at("pooling_kernel_size").integer();
            vc.pos_size = (int)v.at("position_embedding_size").integer();
            vc.eps = (float)v.at("rms_norm_eps").number();
            vc.theta = v.at("rope_parameters").at("rope_theta").number();
            if (v.has("standardize") && v.at("standardize").kind == Json::Bool && v.at("standardize").b)
                fail(EG2_ERR_IO, "vision_config.standardize=true is not supported");
        }
    } catch (Fail&) {
        throw;
    } catch (std::exception& e) {
        fail(EG2_ERR_IO, "config.json: %s", e.what());
    }
}

// ---------------------------------------------------------------------------------------------
// RoPE tables (unique halves): [len, hd / 2], angle = pos * inv_freq[i] in f32 (src/ops.rs:293-314)
// ---------------------------------------------------------------------------------------------
static std::vector<float> rope_inv_freq(double base, int dim) {
    std::vector<float> inv(dim / 2);
    for (int i = 0; i < dim / 2; i++) inv[i] = 1.0f / powf((float)base, (float)(2 * i) / (float)dim);
    return inv;
}

struct RopeTab {
    double theta = 0;
    int hd = 0;
    long len = 0;
    float* cs = nullptr;  // [len, hd / 2]: one position per row (qkv_post: a warp reads one row)
    float* sn = nullptr;
    float* inv = nullptr;  // [hd / 2] inverse frequencies (the fused GEMM epilogue computes its own angles)
};

// ---------------------------------------------------------------------------------------------
// Context
// ---------------------------------------------------------------------------------------------
struct LayerW {
    void *qkv = nullptr, *o = nullptr, *gu = nullptr, *down = nullptr, *pg = nullptr, *pp = nullptr;
    float *input_ln, *post_attn_ln, *pre_ff_ln, *post_ff_ln, *q_norm, *k_norm, *ple_post_norm;
    float layer_scalar = 1.f;
    int hd = 0, nkv = 0, sliding = 0, rope = 0;
    bool qkv_pair = false;  // qkv rows in the pair layout of EPI_QKV_PAIR (bf16, 512-wide heads)
};

struct VLayerW {
    void *qkv = nullptr, *o = nullptr, *gu = nullptr, *down = nullptr;
    float *input_ln, *post_attn_ln, *pre_ff_ln, *post_ff_ln, *q_norm, *k_norm;
};

// Passes of up to kSplitRowsMax rows split the K range of the N = 512 projections into slices (f32
// partial sums, added in slice order by a row kernel), so that the weights are streamed by many SMs:
// unsplit, such a pass has only ceil(rows / 128) two-CTA clusters per projection, each streaming half
// the weight matrix. Up to 8 slices for passes of at most kSplitRowsSmall rows, 4 above (the partial
// sums' traffic grows with rows x slices), never fewer than 2 K blocks per slice. The slice count
// depends only on the row regime and K, so a sequence's bits are the same in any pass of its regime.
constexpr long kSplitRowsSmall = 1024;
constexpr long kSplitRowsMax = 4096;
constexpr long kSplitElems = 16384L * 512;  // partial-sum buffer: slices x rows x 512 (f32)
static int split_slices(long rows, int kb) {
    if (rows > kSplitRowsMax) return 1;
    int S = std::min(rows <= kSplitRowsSmall ? 8 : 4, kb / 2);
    while (S > 1 && kb % S) S--;
    return S >= 2 ? S : 1;
}

struct Work {
    long cap = 0, ple_cap = 0;
    float *hidden = nullptr, *ple = nullptr, *out = nullptr, *x_in = nullptr;
    void *t = nullptr, *qkv = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *a = nullptr, *o = nullptr,
         *gate = nullptr, *pg = nullptr, *gu = nullptr;
    void* xb = nullptr;  // bf16 mode: the pass's input embeddings in bf16 (the PLE projection's input)
    int *pos = nullptr, *seq_start = nullptr, *seq_len = nullptr;
    int* seq_off = nullptr;  // the pass's n_seq + 1 sequence offsets (row_meta expands them per row)
    uint32_t* ids = nullptr;
    long tiles_cap = 0;
    AttnTile* tiles = nullptr;
    long pooled_cap = 0;
    float* pooled = nullptr;
    int* dims = nullptr;
    int seq_meta_cap = 0;
    int* seq_meta = nullptr;
    long pool_scratch_cap = 0;
    double* pool_scratch = nullptr;
    float* osplit = nullptr;  // K-split partial sums of short passes' N = 512 projections [8][256][512]
};

}  // namespace eg2

struct eg2_ctx {
    int device = 0;
    int precision = EG2_BF16;
    std::mutex mu;
    std::string err;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    eg2::TextCfg tc;
    eg2::VisionCfg vc;
    std::vector<void*> allocs;
    // text weights
    std::vector<eg2::LayerW> layers;
    void *ple_proj = nullptr, *emb_proj = nullptr;
    float *ple_norm = nullptr, *final_norm = nullptr;
    uint16_t* embed_table = nullptr;  // bf16 [vocab, hidden] on the device
    bool pre_normed = false;          // this pass's gather also wrote the bf16 input copy and the first pre-norm
    std::vector<eg2::RopeTab> ropes;
    // vision weights
    std::vector<eg2::VLayerW> vlayers;
    void *v_input_proj = nullptr, *v_embed_proj = nullptr;
    float* v_pos_table = nullptr;
    eg2::Work w;
    // vision workspace
    long vcap = 0;
    float *v_hidden = nullptr, *v_pooled = nullptr, *v_cs = nullptr, *v_sn = nullptr, *v_soft = nullptr;
    float* v_inv = nullptr;  // [hd / 4] axial inverse frequencies
    void *v_x = nullptr, *v_t = nullptr, *v_qkv = nullptr, *v_q = nullptr, *v_k = nullptr, *v_v = nullptr, *v_a = nullptr,
         *v_o = nullptr, *v_gate = nullptr, *v_gu = nullptr;
    int *v_pos = nullptr, *v_seq_start = nullptr, *v_seq_len = nullptr;
    eg2::AttnTile* v_tiles = nullptr;            // head-64 attention tiles of the current images
    long v_tiles_cap = 0;
    std::vector<int32_t> v_pos_host;              // positions the RoPE tables in v_cs / v_sn were built for
    int* bad_flag = nullptr;
    // CUDA graphs of short embedding passes (<= 128 rows), one per (row bucket, pooled dims); a graph
    // holds device addresses, so any device (re)allocation (buf_gen) invalidates it.
    struct TextGraph {
        int bucket = 0, n_dims = 0, total = 0;
        uint64_t gen = 0;
        long launches = 0;
        cudaGraphExec_t exec = nullptr;
    };
    std::vector<TextGraph> graphs;
    uint64_t buf_gen = 0;
    cudaStream_t capture_stream = nullptr;
    // profiling
    bool profiling = false;
    std::vector<std::pair<std::string, cudaEvent_t>> marks;
    std::vector<cudaEvent_t> event_pool;
    std::map<std::string, std::pair<double, long>> prof;
    bool use_tc_attention = true;
    // Pass policy. A call is split into passes of at most pass_rows packed rows (a longer sequence
    // gets a pass of its own), consecutive sequences in call order; in bf16 contexts, sequences of at
    // most precise_max tokens run on `precise`, a TF32 context (f32 activations, TF32 GEMMs, f32
    // attention) over the same checkpoint, sharing this context's embedding table and stream.
    long pass_rows = 0;
    int precise_max = 0;
    eg2_ctx* precise = nullptr;
    bool embed_table_shared = false;
    // Multi-pass staging (device): the call's token ids of one pass, and the pooled results of the
    // whole call until every pass has succeeded.
    long stage_ids_cap = 0, stage_out_cap = 0;
    uint32_t* stage_ids = nullptr;
    float* stage_out = nullptr;

    ~eg2_ctx();
};

namespace eg2 {

// Device allocation owned by the context. Buffers a captured graph reads bump buf_gen (the graph holds
// their addresses); staging buffers no graph reads pass graph_visible = false.
static void* dalloc(eg2_ctx* c, size_t bytes, bool graph_visible = true) {
    void* p = nullptr;
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        fail(e == cudaErrorMemoryAllocation ? EG2_ERR_OOM : EG2_ERR_CUDA, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    }
    c->allocs.push_back(p);
    if (graph_visible) c->buf_gen++;
    return p;
}
static void dfree(eg2_ctx* c, void* p, bool graph_visible = true) {
    if (!p) return;
    auto it = std::find(c->allocs.begin(), c->allocs.end(), p);
    if (it != c->allocs.end()) c->allocs.erase(it);
    cudaFree(p);
    if (graph_visible) c->buf_gen++;
}

// Fail before allocating when `need` bytes of device memory are not free, with a message that says what
// to change (the reference's Gpu::ensure_fits, src/gpu/mod.rs:480-505).
static void ensure_fits(size_t need, const char* what, long rows) {
    size_t free_b = 0, total_b = 0;
    CK(cudaMemGetInfo(&free_b, &total_b));
    if (need > free_b) {
        const double gb = 1024.0 * 1024.0 * 1024.0;
        fail(EG2_ERR_OOM,
             "%s for a pass of %ld rows needs about %.1f GB of GPU memory, but %.1f GB of the %.1f GB is free; "
             "lower the pass size (EG2_PASS_ROWS) or the longest sequence",
             what, rows, need / gb, free_b / gb, total_b / gb);
    }
}

static bool bf16_mode(const eg2_ctx* c) { return c->precision == EG2_BF16; }
static size_t act_size(const eg2_ctx* c) { return bf16_mode(c) ? 2 : 4; }

// Upload one weight matrix as the context's GEMM storage (bf16 or f32) into dst (+ row offset).
static void upload_rows(eg2_ctx* c, const SafeTensors& st, const std::string& name, std::initializer_list<long> shape,
                        void* dst, long dst_row0, long row0, long nrows) {
    const TensorInfo& t = st.info(name, shape);
    if (t.dtype != "BF16" && t.dtype != "F32") fail(EG2_ERR_IO, "tensor %s: unsupported dtype", name.c_str());
    const long cols = t.shape.size() >= 2 ? t.shape.back() : 1;
    const uint8_t* src = st.bytes(t);
    const size_t es = act_size(c);
    std::vector<uint8_t> tmp;
    const size_t n = (size_t)nrows * cols;
    if (t.dtype == "BF16" && es == 2) {
        CK(cudaMemcpy((uint8_t*)dst + dst_row0 * cols * 2, src + row0 * cols * 2, n * 2, cudaMemcpyHostToDevice));
        return;
    }
    tmp.resize(n * es);
    for (size_t i = 0; i < n; i++) {
        float f;
        if (t.dtype == "BF16") {
            const uint8_t* b = src + (row0 * cols + i) * 2;
            uint32_t u = (uint32_t)(b[0] | (b[1] << 8)) << 16;
            memcpy(&f, &u, 4);
        } else {
            memcpy(&f, src + (row0 * cols + i) * 4, 4);
        }
        if (es == 4) {
            memcpy(&tmp[i * 4], &f, 4);
        } else {
            uint16_t h = f32_to_bf16_host(f);
            memcpy(&tmp[i * 2], &h, 2);
        }
    }
    CK(cudaMemcpy((uint8_t*)dst + dst_row0 * cols * es, tmp.data(), n * es, cudaMemcpyHostToDevice));
}

// The weight rows of `nheads` 512-channel heads in the pair layout of EPI_QKV_PAIR (kernels.h
// qkv_pair_row): four blocks of 128 rows per head.
static void upload_rows_pair(eg2_ctx* c, const SafeTensors& st, const std::string& name, std::initializer_list<long> shape,
                             void* dst, long dst_row0, long nheads) {
    for (long hh = 0; hh < nheads; hh++)
        for (int np = 0; np < 512; np += 128)
            upload_rows(c, st, name, shape, dst, dst_row0 + hh * 512 + np, hh * 512 + qkv_pair_row(np), 128);
}

static float* upload_vec(eg2_ctx* c, const SafeTensors& st, const std::string& name, long n) {
    std::vector<float> v = st.f32(name, {n});
    float* d = (float*)dalloc(c, n * 4);
    CK(cudaMemcpy(d, v.data(), n * 4, cudaMemcpyHostToDevice));
    return d;
}

// gate|up into one [2 ff, K] matrix, interleaved per 128 features: rows [256 b, 256 b + 128) hold
// gate rows [128 b, 128 b + 128), the next 128 the matching up rows (the EPI_GELU_GU layout).
static void* upload_gate_up(eg2_ctx* c, const SafeTensors& st, const std::string& gate, const std::string& up, long ff,
                            long k) {
    void* d = dalloc(c, 2 * ff * k * act_size(c));
    for (long b = 0; b < ff / 128; b++) {
        upload_rows(c, st, gate, {ff, k}, d, 256 * b, 128 * b, 128);
        upload_rows(c, st, up, {ff, k}, d, 256 * b + 128, 128 * b, 128);
    }
    return d;
}

static void load_text(eg2_ctx* c, const SafeTensors& st) {
    const TextCfg& tc = c->tc;
    const long h = tc.hidden, p = tc.ple, ff = tc.inter, nh = tc.nh;
    if (h % 128 || h > 768 || ff % 128 || p % 256 || tc.emb % 256)
        fail(EG2_ERR_IO, "unsupported text dimensions (hidden %ld, ff %ld, ple %ld)", h, ff, p);
    for (int i = 0; i < tc.layers; i++) {
        LayerW L;
        L.hd = tc.hd[i];
        L.nkv = tc.nkv[i];
        L.sliding = tc.sliding[i];
        const long hd = L.hd, nkv = L.nkv;
        char pre[64];
        snprintf(pre, sizeof pre, "language_model.layers.%d.", i);
        std::string P(pre);
        const long nqkv = (nh + 2 * nkv) * hd;
        L.qkv = dalloc(c, nqkv * h * act_size(c));
        // bf16 with 512-wide heads: rows in the pair layout of the fused QKV epilogue (EPI_QKV_PAIR).
        L.qkv_pair = bf16_mode(c) && hd == 512 && !getenv("EG2_NO_QKV_FUSION");
        if (L.qkv_pair) {
            upload_rows_pair(c, st, P + "self_attn.q_proj.weight", {nh * hd, h}, L.qkv, 0, nh);
            upload_rows_pair(c, st, P + "self_attn.k_proj.weight", {nkv * hd, h}, L.qkv, nh * hd, nkv);
            upload_rows_pair(c, st, P + "self_attn.v_proj.weight", {nkv * hd, h}, L.qkv, (nh + nkv) * hd, nkv);
        } else {
            upload_rows(c, st, P + "self_attn.q_proj.weight", {nh * hd, h}, L.qkv, 0, 0, nh * hd);
            upload_rows(c, st, P + "self_attn.k_proj.weight", {nkv * hd, h}, L.qkv, nh * hd, 0, nkv * hd);
            upload_rows(c, st, P + "self_attn.v_proj.weight", {nkv * hd, h}, L.qkv, (nh + nkv) * hd, 0, nkv * hd);
        }
        L.o = dalloc(c, h * nh * hd * act_size(c));
        upload_rows(c, st, P + "self_attn.o_proj.weight", {h, nh * hd}, L.o, 0, 0, h);
        L.gu = upload_gate_up(c, st, P + "mlp.gate_proj.weight", P + "mlp.up_proj.weight", ff, h);
        L.down = dalloc(c, h * ff * act_size(c));
        upload_rows(c, st, P + "mlp.down_proj.weight", {h, ff}, L.down, 0, 0, h);
        L.pg = dalloc(c, p * h * act_size(c));
        upload_rows(c, st, P + "ple_block.per_layer_input_gate.weight", {p, h}, L.pg, 0, 0, p);
        L.pp = dalloc(c, h * p * act_size(c));
        upload_rows(c, st, P + "ple_block.per_layer_projection.weight", {h, p}, L.pp, 0, 0, h);
        L.input_ln = upload_vec(c, st, P + "input_layernorm.weight", h);
        L.post_attn_ln = upload_vec(c, st, P + "post_attention_layernorm.weight", h);
        L.pre_ff_ln = upload_vec(c, st, P + "pre_feedforward_layernorm.weight", h);
        L.post_ff_ln = upload_vec(c, st, P + "post_feedforward_layernorm.weight", h);
        L.q_norm = upload_vec(c, st, P + "self_attn.q_norm.weight", hd);
        L.k_norm = upload_vec(c, st, P + "self_attn.k_norm.weight", hd);
        L.ple_post_norm = upload_vec(c, st, P + "ple_block.post_per_layer_input_norm.weight", h);
        L.layer_scalar = st.f32(P + "layer_scalar", {1})[0];
        // RoPE table slot per distinct (theta, head_dim), as the reference's rope cache.
        int slot = -1;
        for (size_t r = 0; r < c->ropes.size(); r++)
            if (c->ropes[r].theta == tc.theta[i] && c->ropes[r].hd == L.hd) slot = (int)r;
        if (slot < 0) {
            RopeTab rt;
            rt.theta = tc.theta[i];
            rt.hd = L.hd;
            c->ropes.push_back(rt);
            slot = (int)c->ropes.size() - 1;
        }
        L.rope = slot;
        c->layers.push_back(L);
    }
    c->ple_proj = dalloc(c, (long)tc.layers * p * h * act_size(c));
    upload_rows(c, st, "language_model.ple.per_layer_model_projection.weight", {(long)tc.layers * p, h}, c->ple_proj, 0, 0,
                (long)tc.layers * p);
    c->emb_proj = dalloc(c, (long)tc.emb * h * act_size(c));
    upload_rows(c, st, "language_model.embedding_projection.weight", {(long)tc.emb, h}, c->emb_proj, 0, 0, tc.emb);
    c->ple_norm = upload_vec(c, st, "language_model.ple.per_layer_projection_norm.weight", p);
    c->final_norm = upload_vec(c, st, "language_model.norm.weight", h);
    // Token-embedding table stays bf16 on the device (the device-side gather of eg2_embed_packed).
    const TensorInfo& et = st.info("language_model.embed_tokens.weight", {tc.vocab, h});
    if (et.dtype != "BF16") fail(EG2_ERR_IO, "embed_tokens must be BF16");
    if (c->embed_table) return;  // shared with the context this one serves (see eg2_ctx::precise)
    c->embed_table = (uint16_t*)dalloc(c, (size_t)tc.vocab * h * 2);
    CK(cudaMemcpy(c->embed_table, st.bytes(et), (size_t)tc.vocab * h * 2, cudaMemcpyHostToDevice));
}

static void load_vision(eg2_ctx* c, const SafeTensors& st) {
    VisionCfg& vc = c->vc;
    if (!vc.present || !st.has("vision_tower.patch_embedder.input_proj.weight")) {
        vc.present = false;
        return;
    }
    const long h = vc.hidden, ff = vc.inter, nh = vc.nh, nkv = vc.nkv, hd = vc.hd, pd = 3L * vc.patch * vc.patch;
    if (h % 256 || ff % 128 || pd % 64 || ((nh + 2 * nkv) * hd) % 256 || (nh * hd) % 64) {
        vc.present = false;
        return;
    }
    for (int i = 0; i < vc.layers; i++) {
        VLayerW L;
        char pre[64];
        snprintf(pre, sizeof pre, "vision_tower.encoder.layers.%d.", i);
        std::string P(pre);
        L.qkv = dalloc(c, (nh + 2 * nkv) * hd * h * act_size(c));
        upload_rows(c, st, P + "self_attn.q_proj.linear.weight", {nh * hd, h}, L.qkv, 0, 0, nh * hd);
        upload_rows(c, st, P + "self_attn.k_proj.linear.weight", {nkv * hd, h}, L.qkv, nh * hd, 0, nkv * hd);
        upload_rows(c, st, P + "self_attn.v_proj.linear.weight", {nkv * hd, h}, L.qkv, (nh + nkv) * hd, 0, nkv * hd);
        L.o = dalloc(c, h * nh * hd * act_size(c));
        upload_rows(c, st, P + "self_attn.o_proj.linear.weight", {h, nh * hd}, L.o, 0, 0, h);
        L.gu = upload_gate_up(c, st, P + "mlp.gate_proj.linear.weight", P + "mlp.up_proj.linear.weight", ff, h);
        L.down = dalloc(c, h * ff * act_size(c));
        upload_rows(c, st, P + "mlp.down_proj.linear.weight", {h, ff}, L.down, 0, 0, h);
        L.input_ln = upload_vec(c, st, P + "input_layernorm.weight", h);
        L.post_attn_ln = upload_vec(c, st, P + "post_attention_layernorm.weight", h);
        L.pre_ff_ln = upload_vec(c, st, P + "pre_feedforward_layernorm.weight", h);
        L.post_ff_ln = upload_vec(c, st, P + "post_feedforward_layernorm.weight", h);
        L.q_norm = upload_vec(c, st, P + "self_attn.q_norm.weight", hd);
        L.k_norm = upload_vec(c, st, P + "self_attn.k_norm.weight", hd);
        c->vlayers.push_back(L);
    }
    c->v_input_proj = dalloc(c, h * pd * act_size(c));
    upload_rows(c, st, "vision_tower.patch_embedder.input_proj.weight", {h, pd}, c->v_input_proj, 0, 0, h);
    // The multimodal embedder's projection stays f32 (it runs on the f32 CUDA-core GEMM: N = 512
    // soft-token width is small and the reference runs it on the host in f32).
    {
        std::vector<float> w = st.f32("embed_vision.embedding_projection.weight", {(long)c->tc.hidden, h});
        c->v_embed_proj = dalloc(c, w.size() * 4);
        CK(cudaMemcpy(c->v_embed_proj, w.data(), w.size() * 4, cudaMemcpyHostToDevice));
    }
    std::vector<float> pt = st.f32("vision_tower.patch_embedder.position_embedding_table", {2, (long)vc.pos_size, h});
    c->v_pos_table = (float*)dalloc(c, pt.size() * 4);
    CK(cudaMemcpy(c->v_pos_table, pt.data(), pt.size() * 4, cudaMemcpyHostToDevice));
}

// Grow-only RoPE tables covering positions [0, max_len).
static void ensure_rope(eg2_ctx* c, long max_len) {
    for (RopeTab& r : c->ropes) {
        if (r.len >= max_len) continue;
        long len = ((max_len + 1023) / 1024) * 1024;
        if (len < 4096) len = 4096;
        std::vector<float> inv = rope_inv_freq(r.theta, r.hd);
        const int half = r.hd / 2;
        std::vector<float> cs((size_t)len * half), sn((size_t)len * half);
        for (long t = 0; t < len; t++)
            for (int i = 0; i < half; i++) {
                const float f = (float)t * inv[i];
                cs[(size_t)t * half + i] = cosf(f);
                sn[(size_t)t * half + i] = sinf(f);
            }
        CK(cudaStreamSynchronize(c->stream));
        dfree(c, r.cs);
        dfree(c, r.sn);
        r.cs = (float*)dalloc(c, cs.size() * 4);
        r.sn = (float*)dalloc(c, sn.size() * 4);
        CK(cudaMemcpy(r.cs, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(r.sn, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
        if (!r.inv) {
            r.inv = (float*)dalloc(c, half * 4);
            CK(cudaMemcpy(r.inv, inv.data(), half * 4, cudaMemcpyHostToDevice));
        }
        r.len = len;
    }
}

// Whether a pass of `rows` rows computes each layer's PLE slice inside the PLE-gate GEMM
// (EPI_PLE_FUSED: bf16, above the split-K regime); such a pass needs no [rows, layers, 512] PLE tensor.
static bool ple_fused_pass(const eg2_ctx* c, long rows) {
    return bf16_mode(c) && c->tc.ple == 512 && c->tc.hidden == 512 && split_slices(rows, c->tc.hidden / 64) < 2 &&
           !getenv("EG2_NO_PLE_FUSION");
}

static void ensure_work(eg2_ctx* c, long rows, long n_tiles) {
    Work& w = c->w;
    const TextCfg& tc = c->tc;
    if (rows > w.cap) {
        CK(cudaStreamSynchronize(c->stream));
        long cap = ((rows + 1023) / 1024) * 1024;
        void** bufs[] = {(void**)&w.hidden, (void**)&w.out, (void**)&w.t, (void**)&w.qkv, (void**)&w.q,
                         (void**)&w.k, (void**)&w.v, (void**)&w.a, (void**)&w.o, (void**)&w.gate, (void**)&w.pg,
                         (void**)&w.gu, (void**)&w.pos, (void**)&w.seq_start, (void**)&w.seq_len, (void**)&w.ids,
                         (void**)&w.xb, (void**)&w.seq_off};
        for (void** b : bufs) {
            dfree(c, *b);
            *b = nullptr;
        }
        int max_q = 0, max_kv = 0, max_qkv = 0;
        for (auto& L : c->layers) {
            max_q = std::max(max_q, tc.nh * L.hd);
            max_kv = std::max(max_kv, L.nkv * L.hd);
            max_qkv = std::max(max_qkv, (tc.nh + 2 * L.nkv) * L.hd);
        }
        const size_t as = act_size(c);
        const size_t per_row = (size_t)tc.hidden * 4 + (size_t)tc.emb * 4 + (size_t)tc.hidden * 2 +
                               (size_t)tc.hidden * as + (size_t)max_qkv * 4 + (size_t)(2 * max_q + 2 * max_kv) * as +
                               (size_t)tc.hidden * 4 + (size_t)tc.inter * as + (size_t)tc.ple * as +
                               (c->precision == EG2_F32 ? 2 * (size_t)tc.inter * 4 : 0) + 16;
        ensure_fits(per_row * cap, "the text workspace", rows);
        w.hidden = (float*)dalloc(c, cap * tc.hidden * 4);
        w.out = (float*)dalloc(c, cap * tc.emb * 4);
        w.t = dalloc(c, cap * tc.hidden * as);
        w.qkv = dalloc(c, cap * max_qkv * 4);
        w.q = dalloc(c, cap * max_q * as);
        w.k = dalloc(c, cap * max_kv * as);
        w.v = dalloc(c, cap * max_kv * as);
        w.a = dalloc(c, cap * max_q * as);
        w.o = dalloc(c, cap * tc.hidden * 4);
        w.gate = dalloc(c, cap * tc.inter * as);
        w.pg = dalloc(c, cap * tc.ple * as);
        w.gu = c->precision == EG2_F32 ? dalloc(c, cap * 2L * tc.inter * 4) : nullptr;
        w.xb = bf16_mode(c) ? dalloc(c, cap * tc.hidden * 2) : nullptr;
        w.pos = (int*)dalloc(c, cap * 4);
        w.seq_start = (int*)dalloc(c, cap * 4);
        w.seq_len = (int*)dalloc(c, cap * 4);
        w.seq_off = (int*)dalloc(c, (cap + 1) * 4);
        w.ids = (uint32_t*)dalloc(c, cap * 4);
        w.cap = cap;
    }
    // The PLE tensor [rows, layers, 512] f32 (48 KB per row), only for passes that read it.
    const long ple_rows = ple_fused_pass(c, rows) ? 0 : rows;
    if (ple_rows > w.ple_cap) {
        CK(cudaStreamSynchronize(c->stream));
        dfree(c, w.ple);
        w.ple = nullptr;
        const long cap = ((ple_rows + 1023) / 1024) * 1024;
        const size_t bytes = (size_t)cap * tc.layers * tc.ple * 4;
        ensure_fits(bytes, "the PLE tensor", rows);
        w.ple = (float*)dalloc(c, bytes);
        w.ple_cap = cap;
    }
    if (!w.osplit && (bf16_mode(c) || c->precision == EG2_TF32)) w.osplit = (float*)dalloc(c, (size_t)kSplitElems * 4);
    if (n_tiles > w.tiles_cap) {
        CK(cudaStreamSynchronize(c->stream));
        dfree(c, w.tiles);
        w.tiles_cap = std::max(n_tiles, 1024L);
        w.tiles = (AttnTile*)dalloc(c, w.tiles_cap * sizeof(AttnTile));
    }
}

// ---------------------------------------------------------------------------------------------
// Profiling marks
// ---------------------------------------------------------------------------------------------
static void mark(eg2_ctx* c, const char* label) {
    if (!c->profiling) return;
    cudaEvent_t e;
    if (c->event_pool.empty()) {
        CK(cudaEventCreate(&e));
    } else {
        e = c->event_pool.back();
        c->event_pool.pop_back();
    }
    CK(cudaEventRecord(e, c->stream));
    c->marks.push_back({label, e});
}
static void collect_marks(eg2_ctx* c) {
    if (c->marks.empty()) return;
    CK(cudaEventSynchronize(c->marks.back().second));
    for (size_t i = 1; i < c->marks.size(); i++) {
        float ms = 0;
        cudaEventElapsedTime(&ms, c->marks[i - 1].second, c->marks[i].second);
        auto& p = c->prof[c->marks[i].first];
        p.first += ms;
        p.second += 1;
    }
    for (auto& m : c->marks) c->event_pool.push_back(m.second);
    c->marks.clear();
}

// ---------------------------------------------------------------------------------------------
// GEMM dispatch by precision
// ---------------------------------------------------------------------------------------------
// y = x . W^T with the context's precision. Modes: EPI_STORE (y act, or f32 when out_f32),
// EPI_GELU_GU (y = gelu(gate) * up, N/2 columns), EPI_PLE_GATE (y = gelu(acc) * ple[:, layer]).
static void gemm(eg2_ctx* c, const void* x, long ldx, const void* W, int M, int N, int K, void* y, long ldy, int mode,
                 bool out_f32, float scale = 1.f, const float* aux = nullptr, long aux_ld = 0, int aux_off = 0,
                 void* tmp_f32 = nullptr) {
    if (c->precision == EG2_F32) {
        const float* A = (const float*)x;
        if (mode == EPI_STORE) {
            KL(gemm_f32(A, ldx, (const float*)W, K, (float*)y, ldy, M, N, K, scale, c->stream), "gemm_f32");
        } else if (mode == EPI_GELU_GU) {
            KL(gemm_f32(A, ldx, (const float*)W, K, (float*)tmp_f32, N, M, N, K, 1.f, c->stream), "gemm_f32");
            KL((gelu_gu<float, float>((const float*)tmp_f32, (float*)y, M, N / 2, c->stream)), "gelu_gu");
        } else {
            KL(gemm_f32(A, ldx, (const float*)W, K, (float*)y, ldy, M, N, K, 1.f, c->stream), "gemm_f32");
            KL((ple_gate<float, float>((const float*)y, (float*)y, aux, M, N, c->tc.layers, aux_off / N, c->stream)),
               "ple_gate");
        }
        return;
    }
    GemmEpilogue e;
    e.mode = mode;
    e.out_f32 = out_f32 ? 1 : 0;
    e.out = y;
    e.ldo = ldy;
    e.aux = aux;
    e.aux_ld = aux_ld;
    e.aux_off = aux_off;
    e.scale = scale;
    KL(gemm_tc(bf16_mode(c) ? GEMM_BF16 : GEMM_TF32, x, ldx, W, K, M, N, K, e, c->stream), "gemm_tc");
}

// The q/k/v projection with per-head RMSNorm and RoPE fused into the tensor-core GEMM's epilogue
// (EPI_QKV). Returns false when the configuration does not fuse (f32 precision, or heads that do
// not tile the 256-column output tile); the caller then runs GEMM + qkv_post.
static bool qkv_projection(eg2_ctx* c, const void* x, int k, const void* W, long rows, void* q, void* kk, void* v,
                           const float* wq, const float* wk, const float* inv_freq, const int* pos, int pos_stride, int nh, int nkv, int hd, int part, float eps,
                           bool pair_layout = false) {
    GemmEpilogue e;
    QkvEpilogue& Q = e.qkv;
    Q.q = q, Q.k = kk, Q.v = v, Q.wq = wq, Q.wk = wk, Q.inv_freq = inv_freq, Q.pos = pos, Q.pos_stride = pos_stride;
    Q.nh = nh, Q.nkv = nkv, Q.hd = hd, Q.part = part, Q.eps = eps;
    if (pair_layout) {
        // The weights were loaded in the pair layout: only the fused epilogue undoes it.
        if (!qkv_pair_fusable(Q)) fail(EG2_ERR_INVALID, "qkv pair layout without a fusable configuration");
        e.mode = EPI_QKV_PAIR;
        KL(gemm_tc(GEMM_BF16, x, k, W, k, (int)rows, (nh + 2 * nkv) * hd, k, e, c->stream), "gemm qkv (head 512) + norm/rope");
        mark(c, "gemm qkv (head 512) + norm/rope");
        return true;
    }
    if (c->precision == EG2_F32 || getenv("EG2_NO_QKV_FUSION")) return false;
    e.mode = EPI_QKV;
    if (!qkv_fusable(Q)) return false;
    KL(gemm_tc(bf16_mode(c) ? GEMM_BF16 : GEMM_TF32, x, k, W, k, (int)rows, (nh + 2 * nkv) * hd, k, e, c->stream),
       "gemm qkv + norm/rope");
    mark(c, "gemm qkv + norm/rope");
    return true;
}

// o = x . W^T (N = hidden) followed by the residual update and norms of add_norm():
//   hidden = (hidden + rms_norm(o) * w1) * scalar;  t = w2 ? rms_norm(hidden) * w2 : hidden.
// bf16 with hidden 512 runs it as one GEMM with the EPI_ADD_NORM epilogue (o never leaves the
// tensor memory); otherwise GEMM into w.o (f32) + the add_norm kernel.
template <typename T>
static void gemm_add_norm(eg2_ctx* c, const void* x, long ldx, const void* W, long rows, int K, const float* w1,
                          const float* w2, float scalar, const char* label) {
    Work& w = c->w;
    const int h = c->tc.hidden;
    if (bf16_mode(c) && h == 512 && !getenv("EG2_NO_ADD_NORM_FUSION")) {
        const int S = split_slices(rows, K / 64);
        if (w.osplit && S >= 2 && S * rows <= kSplitElems / h) {
            // A pass of few rows: one cluster per 128-row block would stream the whole weight matrix
            // through few SMs. Split K over S slices instead (S x 2 clusters per 256 rows, f32
            // partials), then sum the partials and update the residual in a row kernel (same
            // arithmetic as the fused epilogue, the sum taken in slice order).
            GemmEpilogue e;
            e.mode = EPI_STORE;
            e.out_f32 = 1;
            e.out = w.osplit;
            e.ldo = h;
            e.ksplit = S;
            e.split_stride = rows * h;
            KL(gemm_tc(GEMM_BF16, x, ldx, W, K, (int)rows, h, K, e, c->stream), label);
            KL(add_norm_split(w.hidden, w.osplit, S, rows * h, w1, (bf16_t*)w.t, w2, rows, h, c->tc.eps, scalar,
                              c->stream),
               "add_norm_split");
            mark(c, label);
            return;
        }
        GemmEpilogue e;
        e.mode = EPI_ADD_NORM;
        e.out = w.t;
        e.ldo = h;
        e.an.h = w.hidden;
        e.an.w1 = w1;
        e.an.w2 = w2;
        e.an.eps = c->tc.eps;
        e.an.scalar = scalar;
        KL(gemm_tc(GEMM_BF16, x, ldx, W, K, (int)rows, h, K, e, c->stream), label);
        mark(c, label);
        return;
    }
    if (c->precision == EG2_TF32 && h == 512 && w.osplit) {
        // TF32 passes of few rows (the short sequences of a bf16 context run here): the K range split into
        // slices as in bf16 (32-element K blocks), f32 partials summed in slice order by the row kernel.
        const int S = split_slices(rows, K / 32);
        if (S >= 2 && S * rows <= kSplitElems / h) {
            GemmEpilogue e;
            e.mode = EPI_STORE;
            e.out_f32 = 1;
            e.out = w.osplit;
            e.ldo = h;
            e.ksplit = S;
            e.split_stride = rows * h;
            KL(gemm_tc(GEMM_TF32, x, ldx, W, K, (int)rows, h, K, e, c->stream), label);
            KL(add_norm_split(w.hidden, w.osplit, S, rows * h, w1, (float*)w.t, w2, rows, h, c->tc.eps, scalar, c->stream),
               "add_norm_split");
            mark(c, label);
            return;
        }
    }
    gemm(c, x, ldx, W, (int)rows, h, K, w.o, h, EPI_STORE, true);
    mark(c, label);
    KL((add_norm<float, T>(w.hidden, (const float*)w.o, w1, (T*)w.t, w2, rows, h, c->tc.eps, scalar, c->stream)), "add_norm");
    mark(c, "add_norm");
}

template <typename T>
static void attention(eg2_ctx* c, const T* q, const T* k, const T* v, T* out, long rows, int nh, int nkv, int hd,
                      int window, const int* seq_start, const int* seq_len, const AttnTile* tiles, int n_tiles);
template <>
void attention<float>(eg2_ctx* c, const float* q, const float* k, const float* v, float* out, long rows, int nh, int nkv,
                      int hd, int window, const int* seq_start, const int* seq_len, const AttnTile*, int) {
    KL(attention_simt<float>(q, k, v, out, seq_start, seq_len, rows, nh, nkv, hd, window, c->stream), "attention_simt");
}
template <>
void attention<bf16_t>(eg2_ctx* c, const bf16_t* q, const bf16_t* k, const bf16_t* v, bf16_t* out, long rows, int nh,
                       int nkv, int hd, int window, const int* seq_start, const int* seq_len, const AttnTile* tiles,
                       int n_tiles) {
    if (c->use_tc_attention && tiles)
        KL(attention_tc(q, k, v, out, rows, tiles, n_tiles, nh, nkv, hd, window, c->stream, seq_start, seq_len),
           "attention_tc");
    else
        KL(attention_simt<bf16_t>(q, k, v, out, seq_start, seq_len, rows, nh, nkv, hd, window, c->stream), "attention_simt");
}

// ---------------------------------------------------------------------------------------------
// Text backbone over w.hidden (rows x hidden f32, already holding the input embeddings).
// Per-layer tile lists: one list per (nkv, head_dim) among the layers.
// ---------------------------------------------------------------------------------------------
struct TileSet {
    int nkv, hd;
    long offset;  // into w.tiles
    int count;
};

template <typename T>
static void enqueue_text(eg2_ctx* c, long rows, const std::vector<TileSet>& tsets) {
    const TextCfg& tc = c->tc;
    Work& w = c->w;
    const int h = tc.hidden, p = tc.ple, nl = tc.layers, nh = tc.nh, ff = tc.inter;
    const float eps = tc.eps;
    const bool f32 = std::is_same<T, float>::value;
    T* t = (T*)w.t;
    mark(c, "set-up + gather");
    // PLE prologue: ple = rmsnorm(embeds . W_ple^T * h^-0.5) * ple_norm per (token, layer) row. Passes
    // above the split-K regime compute each layer's slice inside that layer's PLE-gate GEMM instead
    // (EPI_PLE_FUSED), so the [rows, layers, 512] f32 tensor is never written.
    const bool ple_fused = !f32 && ple_fused_pass(c, rows);
    if (!ple_fused && w.ple_cap < rows) fail(EG2_ERR_INVALID, "PLE tensor smaller than the pass (switch changed between set-up and launch)");
    const void* x_in = w.hidden;
    const bool pre_done = c->pre_normed;  // (embed_gather_norm: w.xb and t are written already)
    c->pre_normed = false;
    if (!f32) {
        if (!pre_done) KL(cast_rows<bf16_t>(w.hidden, (bf16_t*)w.xb, rows * h, 1.f, 0.f, c->stream), "cast");
        x_in = w.xb;
    }
    if (ple_fused) {
        // (nothing here: the slices are computed layer by layer)
    } else if (!f32 && bf16_mode(c) && p == 512) {
        // One GEMM: the per-(token, layer) RMSNorm runs in its epilogue (EPI_GROUP_NORM).
        GemmEpilogue e;
        e.mode = EPI_GROUP_NORM;
        e.out = w.ple;
        e.ldo = (long)nl * p;
        e.scale = powf((float)h, -0.5f);
        e.an.w1 = c->ple_norm;
        e.an.eps = eps;
        KL(gemm_tc(GEMM_BF16, x_in, h, c->ple_proj, h, (int)rows, nl * p, h, e, c->stream), "gemm ple_model + norm");
        mark(c, "gemm ple_model (+ norm)");
    } else {
        gemm(c, x_in, h, c->ple_proj, (int)rows, nl * p, h, w.ple, (long)nl * p, EPI_STORE, true, powf((float)h, -0.5f));
        mark(c, "gemm ple_model");
        KL(rms_norm_inplace(w.ple, c->ple_norm, rows * nl, p, eps, 1.f, c->stream), "rms_norm ple");
    }
    if (!pre_done) KL(rms_norm_rows<T>(w.hidden, t, c->layers[0].input_ln, rows, h, eps, 1.f, c->stream), "rms_norm");
    mark(c, (!f32 && bf16_mode(c) && p == 512) ? "norm (first)" : "norms (ple, first)");
    for (int i = 0; i < nl; i++) {
        const LayerW& L = c->layers[i];
        const int hd = L.hd, nkv = L.nkv;
        const int nqkv = (nh + 2 * nkv) * hd;
        const RopeTab& rt = c->ropes[L.rope];
        const int Sq = split_slices(rows, h / 32);
        if (c->precision == EG2_TF32 && w.osplit && Sq >= 2 && (long)Sq * rows * nqkv <= kSplitElems) {
            // TF32 passes of few rows: the q|k|v projection split over K (f32 partials), then the per-head
            // norm and RoPE with the partials summed in slice order.
            GemmEpilogue e;
            e.mode = EPI_STORE;
            e.out_f32 = 1;
            e.out = w.osplit;
            e.ldo = nqkv;
            e.ksplit = Sq;
            e.split_stride = rows * nqkv;
            KL(gemm_tc(GEMM_TF32, t, h, L.qkv, h, (int)rows, nqkv, h, e, c->stream), "gemm qkv");
            KL(qkv_post_split(w.osplit, Sq, rows * nqkv, (float*)w.q, (float*)w.k, (float*)w.v, L.q_norm, L.k_norm, rt.cs,
                              rt.sn, hd / 2, w.pos, rows, nh, nkv, hd, hd, eps, c->stream),
               "qkv_post");
            mark(c, "gemm qkv + qkv_post (K split)");
        } else if (!qkv_projection(c, t, h, L.qkv, rows, w.q, w.k, w.v, L.q_norm, L.k_norm, rt.inv, w.pos, 1, nh, nkv,
                                   hd, hd, eps, L.qkv_pair)) {
            gemm(c, t, h, L.qkv, (int)rows, nqkv, h, w.qkv, nqkv, EPI_STORE, true);
            mark(c, "gemm qkv");
            KL((qkv_post<float, T>((const float*)w.qkv, (T*)w.q, (T*)w.k, (T*)w.v, L.q_norm, L.k_norm, rt.cs, rt.sn, hd / 2,
                               w.pos, rows, nh, nkv, hd, hd, eps, c->stream)),
               "qkv_post");
            mark(c, "qkv_post");
        }
        const AttnTile* tiles = nullptr;
        int n_tiles = 0;
        for (const TileSet& s : tsets)
            if (s.nkv == nkv && s.hd == hd) {
                tiles = w.tiles + s.offset;
                n_tiles = s.count;
            }
        attention<T>(c, (const T*)w.q, (const T*)w.k, (const T*)w.v, (T*)w.a, rows, nh, nkv, hd,
                     L.sliding ? tc.window : -1, w.seq_start, w.seq_len, tiles, n_tiles);
        mark(c, hd == 256 ? "attention d256" : "attention d512");
        gemm_add_norm<T>(c, w.a, nh * hd, L.o, rows, nh * hd, L.post_attn_ln, L.pre_ff_ln, 1.f, "gemm o (+ add_norm)");
        if (c->precision == EG2_TF32 && w.osplit && Sq >= 2 && (long)Sq * rows * 2 * ff <= kSplitElems) {
            // TF32 passes of few rows: gate|up split over K, then gelu(gate) * up over the summed partials.
            GemmEpilogue e;
            e.mode = EPI_STORE;
            e.out_f32 = 1;
            e.out = w.osplit;
            e.ldo = 2 * ff;
            e.ksplit = Sq;
            e.split_stride = rows * 2L * ff;
            KL(gemm_tc(GEMM_TF32, t, h, L.gu, h, (int)rows, 2 * ff, h, e, c->stream), "gemm gate|up");
            KL(gelu_gu_split(w.osplit, Sq, rows * 2L * ff, (float*)w.gate, rows, ff, c->stream), "gelu_gu_split");
        } else {
            gemm(c, t, h, L.gu, (int)rows, 2 * ff, h, w.gate, ff, EPI_GELU_GU, f32, 1.f, nullptr, 0, 0, w.gu);
        }
        mark(c, "gemm gate|up + gelu");
        // t = hidden (as the per-layer-input gate's input, bf16 in bf16 mode).
        gemm_add_norm<T>(c, w.gate, ff, L.down, rows, ff, L.post_ff_ln, nullptr, 1.f, "gemm down (+ add_norm)");
        const int Sg = split_slices(rows, h / 64);
        const int Sg32 = split_slices(rows, h / 32);  // TF32: 32-element K blocks
        if (ple_fused) {
            KL(gemm_ple_fused((const bf16_t*)t, (const bf16_t*)w.xb, (const bf16_t*)L.pg, (const bf16_t*)c->ple_proj, i,
                              c->ple_norm, powf((float)h, -0.5f), eps, (bf16_t*)w.pg, (int)rows, c->stream),
               "gemm ple_gate + ple slice");
        } else if (bf16_mode(c) && Sg >= 2 && w.osplit && p == 512 && h % 128 == 0 && Sg * rows <= kSplitElems / p) {
            // A pass of few rows: the K range split into slices (f32 partials), then GELU x ple in a
            // row kernel.
            GemmEpilogue e;
            e.mode = EPI_STORE;
            e.out_f32 = 1;
            e.out = w.osplit;
            e.ldo = p;
            e.ksplit = Sg;
            e.split_stride = rows * p;
            KL(gemm_tc(GEMM_BF16, t, h, L.pg, h, (int)rows, p, h, e, c->stream), "gemm ple_gate");
            KL(ple_gate_split(w.osplit, Sg, rows * p, w.ple, (long)nl * p, i * p, (bf16_t*)w.pg, rows, p, c->stream),
               "ple_gate_split");
        } else if (c->precision == EG2_TF32 && Sg32 >= 2 && w.osplit && p == 512 && Sg32 * rows <= kSplitElems / p) {
            // The same for TF32 passes of few rows (f32 gate output).
            GemmEpilogue e;
            e.mode = EPI_STORE;
            e.out_f32 = 1;
            e.out = w.osplit;
            e.ldo = p;
            e.ksplit = Sg32;
            e.split_stride = rows * p;
            KL(gemm_tc(GEMM_TF32, t, h, L.pg, h, (int)rows, p, h, e, c->stream), "gemm ple_gate");
            KL(ple_gate_split(w.osplit, Sg32, rows * p, w.ple, (long)nl * p, i * p, (float*)w.pg, rows, p, c->stream),
               "ple_gate_split");
        } else {
            gemm(c, t, h, L.pg, (int)rows, p, h, w.pg, p, EPI_PLE_GATE, f32, 1.f, w.ple, (long)nl * p, i * p);
        }
        mark(c, "gemm ple_gate");
        const float* next_w = (i + 1 < nl) ? c->layers[i + 1].input_ln : c->final_norm;
        gemm_add_norm<T>(c, w.pg, p, L.pp, rows, p, L.ple_post_norm, next_w, L.layer_scalar, "gemm ple_proj (+ add_norm)");
    }
    gemm(c, t, h, c->emb_proj, (int)rows, tc.emb, h, w.out, tc.emb, EPI_STORE, true);
    mark(c, "gemm embed_proj");
}

// Row metadata and attention tile lists for sequences packed back to back. tile_slots > 0 pads each
// tile list to that many entries with empty tiles (length 0: the attention CTAs exit at once), so a
// captured graph's grid sizes stay valid for any sequence split of the same row count.
static std::vector<TileSet> prepare_pass(eg2_ctx* c, const int32_t* lens, int n_seq, long rows, int tile_slots = 0) {
    const TextCfg& tc = c->tc;
    c->pre_normed = false;
    // Sequence offsets only: the per-row position and sequence bounds are expanded on the device.
    std::vector<int> off(n_seq + 1);
    long max_len = 0;
    off[0] = 0;
    for (int s = 0; s < n_seq; s++) {
        off[s + 1] = off[s] + lens[s];
        max_len = std::max<long>(max_len, lens[s]);
    }
    std::vector<std::pair<int, int>> kinds;  // (nkv, head_dim) of the layers
    for (auto& L : c->layers) {
        const std::pair<int, int> kd(L.nkv, L.hd);
        if (std::find(kinds.begin(), kinds.end(), kd) == kinds.end()) kinds.push_back(kd);
    }
    std::vector<TileSet> sets;
    std::vector<AttnTile> tiles;
    if (bf16_mode(c) && c->use_tc_attention) {
        for (const auto& kd : kinds) {
            TileSet ts;
            ts.nkv = kd.first;
            ts.hd = kd.second;
            ts.offset = (long)tiles.size();
            const int tq = attention_tc_tile_tokens(tc.nh, kd.first, kd.second);
            // A sequence of tq tokens or more gets its own tiles. Shorter ones share a tile with their
            // short neighbours while the group fits in tq rows: the tile spans the group's rows and each
            // row masks the keys outside its own sequence (the kernel reads the per-row sequence
            // bounds), so a batch of short queries takes few tiles instead of one per query.
            long row0 = 0;
            int g_row0 = 0, g_rows = 0;  // open group of short sequences
            auto close_group = [&]() {
                if (g_rows > 0) tiles.push_back(AttnTile{g_row0, g_rows, 0});
                g_rows = 0;
            };
            for (int s = 0; s < n_seq; s++) {
                if (lens[s] < tq) {
                    if (g_rows + lens[s] > tq) close_group();
                    if (g_rows == 0) g_row0 = (int)row0;
                    g_rows += lens[s];
                } else {
                    close_group();
                    for (int q0 = 0; q0 < lens[s]; q0 += tq) tiles.push_back(AttnTile{(int)row0, lens[s], q0});
                }
                row0 += lens[s];
            }
            close_group();
            if (tile_slots > 0) {
                if ((long)tiles.size() - ts.offset > tile_slots) fail(EG2_ERR_INVALID, "tile list exceeds its slots");
                while ((long)tiles.size() - ts.offset < tile_slots) tiles.push_back(AttnTile{0, 0, 0});
            }
            ts.count = (int)(tiles.size() - ts.offset);
            sets.push_back(ts);
        }
    }
    ensure_work(c, rows, (long)tiles.size());
    ensure_rope(c, max_len);
    Work& w = c->w;
    CK(cudaMemcpyAsync(w.seq_off, off.data(), (size_t)(n_seq + 1) * 4, cudaMemcpyHostToDevice, c->stream));
    KL(row_meta(w.seq_off, n_seq, rows, w.pos, w.seq_start, w.seq_len, c->stream), "row_meta");
    if (!tiles.empty())
        CK(cudaMemcpyAsync(w.tiles, tiles.data(), tiles.size() * sizeof(AttnTile), cudaMemcpyHostToDevice, c->stream));
    // The host vectors die at return: make the copies complete first.
    CK(cudaStreamSynchronize(c->stream));
    return sets;
}

static long check_lens(const int32_t* lens, int n_seq) {
    if (n_seq < 0 || (n_seq > 0 && !lens)) fail(EG2_ERR_INVALID, "bad sequence list");
    long rows = 0;
    for (int s = 0; s < n_seq; s++) {
        if (lens[s] <= 0) fail(EG2_ERR_INVALID, "empty token sequence (index %d)", s);
        rows += lens[s];
    }
    if (rows > (1L << 30)) fail(EG2_ERR_INVALID, "too many rows");
    return rows;
}

static void check_device_status(eg2_ctx* c) {
    int st = 0;
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaMemcpyFromSymbol(&st, eg2_dev_status, sizeof(int)));
    if (st) {
        int zero = 0;
        cudaMemcpyToSymbol(eg2_dev_status, &zero, sizeof(int));
        fail(EG2_ERR_TIMEOUT, "a device-side wait ran out (code %d)", st);
    }
}

static void run_text(eg2_ctx* c, long rows, const std::vector<TileSet>& sets) {
    if (bf16_mode(c))
        enqueue_text<bf16_t>(c, rows, sets);
    else
        enqueue_text<float>(c, rows, sets);
}

// ---------------------------------------------------------------------------------------------
// Vision tower (src/vision.rs:223-273)
// ---------------------------------------------------------------------------------------------
template <typename T>
// n rows: the patches of n_img images of gh x gw patches each, image after image (so the images stack
// along the patch rows: a gh-row band per image, and pooling windows never cross two images).
static void enqueue_vision(eg2_ctx* c, long n, int gh, int gw, int n_img, int n_tiles) {
    const VisionCfg& vc = c->vc;
    const int h = vc.hidden, ff = vc.inter, nh = vc.nh, nkv = vc.nkv, hd = vc.hd, pd = 3 * vc.patch * vc.patch;
    const bool f32 = std::is_same<T, float>::value;
    const float eps = vc.eps;
    T* t = (T*)c->v_t;
    mark(c, "start");
    // v_t holds 2 (x - 0.5) in the GEMM storage type (written by the caller).
    gemm(c, c->v_t, pd, c->v_input_proj, (int)n, h, pd, c->v_hidden, h, EPI_STORE, true);
    KL(vision_add_positions(c->v_hidden, c->v_pos_table, c->v_pos, n, h, vc.pos_size, c->stream), "positions");
    mark(c, "vision input");
    KL(rms_norm_rows<T>(c->v_hidden, t, c->vlayers[0].input_ln, n, h, eps, 1.f, c->stream), "rms_norm");
    const int nqkv = (nh + 2 * nkv) * hd;
    // bf16 with 768-wide rows: the O and down projections end in the add-norm epilogue (as the text
    // tower's, on clusters of three CTAs): 32 images of 2,304 patches in one call 1.38 -> 1.29 ms per
    // image; one image per call 1-2% slower (18 clusters of three), kept fused so that an image gives the
    // same bits alone or in a batch. EG2_NO_ADD_NORM_FUSION=1 keeps GEMM + add_norm kernel.
    const bool fuse_an = bf16_mode(c) && h == 768 && !getenv("EG2_NO_ADD_NORM_FUSION");
    for (int l = 0; l < vc.layers; l++) {
        const VLayerW& L = c->vlayers[l];
        if (!qkv_projection(c, t, h, L.qkv, n, c->v_q, c->v_k, c->v_v, L.q_norm, L.k_norm, c->v_inv, c->v_pos, 2,
                            nh, nkv, hd, hd / 2, eps)) {
            gemm(c, t, h, L.qkv, (int)n, nqkv, h, c->v_qkv, nqkv, EPI_STORE, true);
            KL((qkv_post<float, T>((const float*)c->v_qkv, (T*)c->v_q, (T*)c->v_k, (T*)c->v_v, L.q_norm, L.k_norm, c->v_cs,
                               c->v_sn, hd / 2, nullptr, n, nh, nkv, hd, hd / 2, eps, c->stream)),
               "qkv_post");
        }
        mark(c, "vision qkv");
        if (f32)
            KL(attention_simt<float>((const float*)c->v_q, (const float*)c->v_k, (const float*)c->v_v, (float*)c->v_a,
                                     c->v_seq_start, c->v_seq_len, n, nh, nkv, hd, -1, c->stream),
               "attention");
        else if (attention_tc_tile_tokens(nh, nkv, hd) == 256 && hd == 64)
            KL(attention_tc((const bf16_t*)c->v_q, (const bf16_t*)c->v_k, (const bf16_t*)c->v_v, (bf16_t*)c->v_a, n,
                            c->v_tiles, n_tiles, nh, nkv, hd, -1, c->stream),
               "attention_tc");
        else
            KL(attention_simt<bf16_t>((const bf16_t*)c->v_q, (const bf16_t*)c->v_k, (const bf16_t*)c->v_v, (bf16_t*)c->v_a,
                                      c->v_seq_start, c->v_seq_len, n, nh, nkv, hd, -1, c->stream),
               "attention");
        mark(c, "vision attention");
        const float* next_w = (l + 1 < vc.layers) ? c->vlayers[l + 1].input_ln : nullptr;
        if (fuse_an) {
            // The residual update and norms in the O / down GEMMs' epilogue (clusters of three CTAs over the
            // 768-wide rows); t is written even after the last layer (unread).
            auto an_gemm = [&](const void* x, int K, const void* W, const float* w1, const float* w2, const char* label) {
                GemmEpilogue e;
                e.mode = EPI_ADD_NORM;
                e.out = t;
                e.ldo = h;
                e.an.h = c->v_hidden;
                e.an.w1 = w1;
                e.an.w2 = w2;
                e.an.eps = eps;
                e.an.scalar = 1.f;
                KL(gemm_tc(GEMM_BF16, x, K, W, K, (int)n, h, K, e, c->stream), label);
                mark(c, label);
            };
            an_gemm(c->v_a, nh * hd, L.o, L.post_attn_ln, L.pre_ff_ln, "vision gemm o (+ add_norm)");
            gemm(c, t, h, L.gu, (int)n, 2 * ff, h, c->v_gate, ff, EPI_GELU_GU, f32, 1.f, nullptr, 0, 0, c->v_gu);
            mark(c, "vision gemm gate|up + gelu");
            an_gemm(c->v_gate, ff, L.down, L.post_ff_ln, next_w, "vision gemm down (+ add_norm)");
            continue;
        }
        gemm(c, c->v_a, nh * hd, L.o, (int)n, h, nh * hd, c->v_o, h, EPI_STORE, true);
        mark(c, "vision gemm o");
        KL((add_norm<float, T>(c->v_hidden, (const float*)c->v_o, L.post_attn_ln, t, L.pre_ff_ln, n, h, eps, 1.f, c->stream)), "add_norm");
        mark(c, "vision add_norm");
        gemm(c, t, h, L.gu, (int)n, 2 * ff, h, c->v_gate, ff, EPI_GELU_GU, f32, 1.f, nullptr, 0, 0, c->v_gu);
        mark(c, "vision gemm gate|up + gelu");
        gemm(c, c->v_gate, ff, L.down, (int)n, h, ff, c->v_o, h, EPI_STORE, true);
        mark(c, "vision gemm down");
        KL((add_norm<float, T>(c->v_hidden, (const float*)c->v_o, L.post_ff_ln, next_w ? t : (T*)nullptr, next_w, n, h, eps, 1.f,
                           c->stream)),
           "add_norm");
        mark(c, "vision add_norm");
    }
    const long oh = (long)n_img * (gh / vc.pool), ow = gw / vc.pool;
    KL(vision_pool(c->v_hidden, c->v_pooled, (int)(n_img * gh), gw, h, vc.pool, sqrtf((float)h), c->stream), "vision_pool");
    // Multimodal embedder: scale-free RMSNorm, then 768 -> text hidden (src/vision.rs:167-170; f32 on the
    // reference's host). f32 mode keeps the f32 CUDA-core GEMM; the tensor-core modes run it as a TF32
    // tcgen05 GEMM on the f32 weights (10-bit mantissa inputs, f32 accumulation).
    float* normed = (float*)c->v_o;  // reuse: oh*ow*h f32 fits (act buffer sized n*h*4)
    KL(rms_norm_rows<float>(c->v_pooled, normed, nullptr, oh * ow, h, eps, 1.f, c->stream), "rms_norm");
    if (f32 && c->precision == EG2_F32) {
        KL(gemm_f32(normed, h, (const float*)c->v_embed_proj, h, c->v_soft, c->tc.hidden, (int)(oh * ow), c->tc.hidden, h,
                    1.f, c->stream),
           "gemm_f32");
    } else {
        GemmEpilogue e;
        e.mode = EPI_STORE;
        e.out_f32 = 1;
        e.out = c->v_soft;
        e.ldo = c->tc.hidden;
        KL(gemm_tc(GEMM_TF32, normed, h, c->v_embed_proj, h, (int)(oh * ow), c->tc.hidden, h, e, c->stream), "gemm_tc tf32");
    }
    mark(c, "vision pool + embed");
}

}  // namespace eg2

using namespace eg2;

eg2_ctx::~eg2_ctx() {
    if (stream) cudaStreamSynchronize(stream);
    delete precise;
    for (auto& g : graphs)
        if (g.exec) cudaGraphExecDestroy(g.exec);
    if (capture_stream) cudaStreamDestroy(capture_stream);
    for (void* p : allocs) cudaFree(p);
    for (auto& m : marks) cudaEventDestroy(m.second);
    for (auto e : event_pool) cudaEventDestroy(e);
    if (own_stream) cudaStreamDestroy(own_stream);
}

static thread_local std::string g_open_error;

template <typename F>
static int guarded(eg2_ctx* c, F&& f) {
    if (!c) return EG2_ERR_INVALID;
    std::lock_guard<std::mutex> lk(c->mu);
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != c->device) cudaSetDevice(c->device);
    int rc = EG2_OK;
    try {
        f();
    } catch (Fail& e) {
        c->err = e.msg;
        rc = e.code;
        c->marks.clear();
    } catch (std::exception& e) {
        c->err = e.what();
        rc = EG2_ERR_INVALID;
    }
    if (prev != c->device) cudaSetDevice(prev);
    return rc;
}

extern "C" {

}  // extern "C"

// Rows of one device pass: 64 documents of 2,208 tokens (141,312 rows, the throughput plateau on a
// B200 at ~11 GB of bf16 workspace) plus room for a slightly larger pack. EG2_PASS_ROWS overrides.
constexpr long kPassRowsDefault = 147456;
// Sequences of at most this many tokens run in TF32 inside bf16 contexts. Their bf16 rounding errors
// are not averaged over many tokens by the mean pool: measured on the random-init checkpoint, 1-5-token
// documents reach 3.4e-3 to 4.3e-3 max-abs against the f32 oracle in bf16 (the bf16 profile allows
// 4e-3), 17-token ones 2.8e-3, and TF32 stays near 5e-4. EG2_PRECISE_MAX_TOKENS overrides (0: off).
constexpr int kPreciseMaxDefault = 16;

static long env_long(const char* name, long dflt, long lo, long hi) {
    const char* e = getenv(name);
    if (!e || !*e) return dflt;
    char* end = nullptr;
    const long v = strtol(e, &end, 10);
    if (end == e || v < lo || v > hi) return dflt;
    return v;
}

// Open one context. text_only skips the vision tower; shared_table (device, bf16) is used as the
// token-embedding table instead of uploading a copy.
static int open_ctx(int device, int precision, const std::string& dir, bool text_only, uint16_t* shared_table,
                    eg2_ctx** out) {
    eg2_ctx* c = new eg2_ctx();
    c->device = device;
    c->precision = precision;
    c->pass_rows = env_long("EG2_PASS_ROWS", kPassRowsDefault, 1024, 1L << 30);
    try {
        CK(cudaSetDevice(device));
        int major = 0, minor = 0;
        CK(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
        CK(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
        if (major != 10 || minor != 0) fail(EG2_ERR_CUDA, "device %d is sm_%d%d; this library is built for sm_100a", device, major, minor);
        CK(cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking));
        c->stream = c->own_stream;
        parse_config(dir, c->tc, c->vc);
        if (text_only) c->vc.present = false;
        SafeTensors st(dir + "/model.safetensors");
        if (shared_table) {
            c->embed_table = shared_table;
            c->embed_table_shared = true;
        }
        load_text(c, st);
        load_vision(c, st);
        c->bad_flag = (int*)dalloc(c, 4);
        CK(cudaMemset(c->bad_flag, 0, 4));
        const char* env = getenv("EG2_SIMT_ATTENTION");
        if (env && env[0] == '1') c->use_tc_attention = false;
        if (precision == EG2_BF16 && !text_only) {
            c->precise_max = (int)env_long("EG2_PRECISE_MAX_TOKENS", kPreciseMaxDefault, 0, 4096);
            if (c->precise_max > 0) {
                const int rc = open_ctx(device, EG2_TF32, dir, true, c->embed_table, &c->precise);
                if (rc != EG2_OK) fail(rc, "opening the TF32 context for short sequences: %s", g_open_error.c_str());
            }
        }
        CK(cudaDeviceSynchronize());
    } catch (Fail& e) {
        g_open_error = e.msg;
        delete c;
        return e.code;
    } catch (std::exception& e) {
        g_open_error = e.what();
        delete c;
        return EG2_ERR_IO;
    }
    *out = c;
    return EG2_OK;
}

extern "C" {

int eg2_open(int device, int precision, const char* model_dir, eg2_ctx** out) {
    if (!out || !model_dir || precision < EG2_F32 || precision > EG2_BF16) {
        g_open_error = "invalid argument";
        return EG2_ERR_INVALID;
    }
    *out = nullptr;
    int prev = 0;
    cudaGetDevice(&prev);
    eg2_ctx* c = nullptr;
    const int rc = open_ctx(device, precision, std::string(model_dir), false, nullptr, &c);
    cudaSetDevice(prev);
    if (rc == EG2_OK) *out = c;
    return rc;
}

void eg2_close(eg2_ctx* c) {
    if (!c) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(c->device);
    delete c;
    cudaSetDevice(prev);
}

const char* eg2_last_error(const eg2_ctx* c) { return c ? c->err.c_str() : g_open_error.c_str(); }

int eg2_text_dims(const eg2_ctx* c, int* hidden, int* emb, int64_t* vocab, int* layers) {
    if (!c) return EG2_ERR_INVALID;
    if (hidden) *hidden = c->tc.hidden;
    if (emb) *emb = c->tc.emb;
    if (vocab) *vocab = c->tc.vocab;
    if (layers) *layers = c->tc.layers;
    return EG2_OK;
}

int eg2_set_stream(eg2_ctx* c, void* stream) {
    return guarded(c, [&] {
        CK(cudaStreamSynchronize(c->stream));
        c->stream = stream ? (cudaStream_t)stream : c->own_stream;
    });
}

int eg2_embed_tokens(eg2_ctx* c, const uint32_t* ids, int64_t n, float* out) {
    return guarded(c, [&] {
        if (n < 0 || (n > 0 && (!ids || !out))) fail(EG2_ERR_INVALID, "bad arguments");
        if (n == 0) return;
        for (int64_t i = 0; i < n; i++)
            if ((int64_t)ids[i] >= c->tc.vocab) fail(EG2_ERR_INVALID, "token id %u out of range", ids[i]);
        // In chunks of at most one pass's rows, so the workspace stays bounded for any n.
        const long chunk = std::min<long>(n, c->pass_rows);
        ensure_work(c, chunk, 0);
        Work& w = c->w;
        const int h = c->tc.hidden;
        for (int64_t i0 = 0; i0 < n; i0 += chunk) {
            const long m = std::min<long>(chunk, n - i0);
            CK(cudaMemcpyAsync(w.ids, ids + i0, m * 4, cudaMemcpyHostToDevice, c->stream));
            KL(embed_gather(c->embed_table, c->tc.vocab, h, w.ids, m, sqrtf((float)h), w.hidden, c->bad_flag, c->stream),
               "embed_gather");
            CK(cudaMemcpyAsync(out + i0 * h, w.hidden, m * h * 4, cudaMemcpyDeviceToHost, c->stream));
        }
        CK(cudaStreamSynchronize(c->stream));
    });
}

// ---------------------------------------------------------------------------------------------
// Pass policy (the reference's embed_prepared packs consecutive inputs greedily into passes of at
// most PACK_TOKENS = 2,048 rows, a longer sequence forming a pass of its own, src/model.rs:157-158,
// :508-521). Here the cap is sized for a B200 (one 64 x 2,208-token pass, the throughput plateau,
// with ~11 GB of workspace), so one call of any size runs in a bounded workspace; and in bf16
// contexts the sequences of at most `precise_max` tokens form their own passes on the TF32 context.
// A pass is a set of consecutive sequences of one class in call order, so its results are the same
// bits as a call holding only those sequences.
// ---------------------------------------------------------------------------------------------
struct Pass {
    std::vector<int> seqs;  // the call's sequence indices, ascending
    long rows = 0;
    bool precise = false;
};

static std::vector<Pass> plan_passes(const int32_t* lens, int n_seq, long max_rows, int precise_max) {
    std::vector<Pass> done;
    Pass open[2];
    open[1].precise = true;
    for (int s = 0; s < n_seq; s++) {
        const int k = (precise_max > 0 && lens[s] <= precise_max) ? 1 : 0;
        if (!open[k].seqs.empty() && open[k].rows + lens[s] > max_rows) {
            done.push_back(std::move(open[k]));
            open[k] = Pass();
            open[k].precise = k == 1;
        }
        open[k].seqs.push_back(s);
        open[k].rows += lens[s];
    }
    for (int k = 0; k < 2; k++)
        if (!open[k].seqs.empty()) done.push_back(std::move(open[k]));
    return done;
}

// Sequences of a pass that are consecutive in the call: call sequences [seq0, seq0 + nseq), the
// pass's sequences [pseq0, ...), call rows [row0, row0 + rows) at pass row prow0.
struct Run {
    int seq0, nseq, pseq0;
    long row0, prow0, rows;
};

static std::vector<Run> pass_runs(const Pass& p, const std::vector<long>& seq_row0, const int32_t* lens) {
    std::vector<Run> runs;
    long prow = 0;
    for (size_t i = 0; i < p.seqs.size(); i++) {
        const int s = p.seqs[i];
        if (!runs.empty() && runs.back().seq0 + runs.back().nseq == s) {
            runs.back().nseq++;
            runs.back().rows += lens[s];
        } else {
            runs.push_back(Run{s, 1, (int)i, seq_row0[s], prow, (long)lens[s]});
        }
        prow += lens[s];
    }
    return runs;
}

static std::vector<long> row_offsets(const int32_t* lens, int n_seq) {
    std::vector<long> r0(n_seq);
    long r = 0;
    for (int s = 0; s < n_seq; s++) {
        r0[s] = r;
        r += lens[s];
    }
    return r0;
}

// The passes of a call on context c (the TF32 context takes the short sequences of bf16 contexts).
static std::vector<Pass> call_plan(eg2_ctx* c, const int32_t* lens, int n_seq) {
    const int pmax = (c->precise && bf16_mode(c)) ? c->precise_max : 0;
    if (c->precise) c->precise->stream = c->stream;
    return plan_passes(lens, n_seq, c->pass_rows, pmax);
}

// Grow-only staging buffers of the parent context (no captured graph reads them).
static void ensure_stage(eg2_ctx* c, long ids_rows, long out_floats) {
    if (ids_rows > c->stage_ids_cap) {
        CK(cudaStreamSynchronize(c->stream));
        dfree(c, c->stage_ids, false);
        c->stage_ids = nullptr;
        c->stage_ids_cap = std::max(ids_rows, 4096L);
        c->stage_ids = (uint32_t*)dalloc(c, c->stage_ids_cap * 4, false);
    }
    if (out_floats > c->stage_out_cap) {
        CK(cudaStreamSynchronize(c->stream));
        dfree(c, c->stage_out, false);
        c->stage_out = nullptr;
        c->stage_out_cap = std::max(out_floats, 4096L);
        c->stage_out = (float*)dalloc(c, c->stage_out_cap * 4, false);
    }
}

static int forward_impl(eg2_ctx* c, const float* embeds, const int32_t* lens, int n_seq, float* out, void* stream,
                        bool device_ptrs) {
    return guarded(c, [&] {
        cudaStream_t saved = c->stream;
        if (stream) c->stream = (cudaStream_t)stream;
        struct Restore {
            eg2_ctx* c;
            cudaStream_t s;
            ~Restore() { c->stream = s; }
        } restore{c, saved};
        const long rows = check_lens(lens, n_seq);
        if (rows == 0) return;
        if (!embeds || !out) fail(EG2_ERR_INVALID, "null buffer");
        const int h = c->tc.hidden, emb = c->tc.emb;
        const cudaMemcpyKind in_kind = device_ptrs ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
        const cudaMemcpyKind out_kind = device_ptrs ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
        const auto plan = call_plan(c, lens, n_seq);
        const auto seq_row0 = row_offsets(lens, n_seq);
        // Each pass runs, is checked, then writes its rows of `out`: an argument error leaves `out`
        // untouched; a device failure in a later pass of a multi-pass call leaves the rows of the passes
        // before it written.
        for (const Pass& p : plan) {
            eg2_ctx* x = p.precise ? c->precise : c;
            const auto runs = pass_runs(p, seq_row0, lens);
            std::vector<int32_t> plens;
            for (int s : p.seqs) plens.push_back(lens[s]);
            // The pass's embeddings into x's workspace, then its 24 layers; the per-token states land in x->w.out.
            const auto sets = prepare_pass(x, plens.data(), (int)plens.size(), p.rows);
            for (const Run& r : runs)
                CK(cudaMemcpyAsync(x->w.hidden + r.prow0 * h, embeds + r.row0 * h, r.rows * h * 4, in_kind, c->stream));
            run_text(x, p.rows, sets);
            check_device_status(c);
            collect_marks(c);
            for (const Run& r : runs)
                CK(cudaMemcpyAsync(out + r.row0 * emb, x->w.out + r.prow0 * emb, r.rows * emb * 4, out_kind, c->stream));
        }
        CK(cudaStreamSynchronize(c->stream));
    });
}

int eg2_forward_packed(eg2_ctx* c, const float* embeds, const int32_t* lens, int n_seq, float* out) {
    return forward_impl(c, embeds, lens, n_seq, out, nullptr, false);
}
int eg2_forward_packed_device(eg2_ctx* c, const float* embeds, const int32_t* lens, int n_seq, float* out, void* stream) {
    return forward_impl(c, embeds, lens, n_seq, out, stream, true);
}

// Short passes (<= 128 rows, bf16 or TF32): rows are padded to a bucket of 16 / 32 / 64 / 128 with one
// extra sequence of token 0, the attention tile lists and the pooled-sequence list to bucket + 1
// entries (empty ones have length 0), so every launch of the pass has the same parameters for any
// split of the bucket into sequences. The pass (gather, 24 layers, pool) is captured once per
// (bucket, dims) into a CUDA graph and replayed with new metadata: ~175 launches become one (the
// reference captures graphs per row bucket for the same reason, src/gpu/text.rs:475-516). The pooled
// results are left in c->w.pooled.
// The gather of a text pass's embeddings; bf16 contexts with 512-wide rows also write the bf16 input
// copy and the first pre-norm in the same kernel (enqueue_text then skips them).
static void gather_pass(eg2_ctx* c, long rows) {
    Work& w = c->w;
    const int h = c->tc.hidden;
    if (bf16_mode(c) && h == 512) {
        KL(embed_gather_norm(c->embed_table, c->tc.vocab, h, w.ids, rows, sqrtf((float)h), w.hidden, (bf16_t*)w.xb,
                             (bf16_t*)w.t, c->layers[0].input_ln, c->tc.eps, c->bad_flag, c->stream),
           "embed_gather_norm");
        c->pre_normed = true;
    } else {
        KL(embed_gather(c->embed_table, c->tc.vocab, h, w.ids, rows, sqrtf((float)h), w.hidden, c->bad_flag, c->stream),
           "embed_gather");
    }
}

static void embed_graph(eg2_ctx* c, const uint32_t* ids, const int32_t* lens, int n_seq, long rows, const int32_t* dims,
                        int n_dims, int total, bool ids_on_device) {
    const int B = rows <= 16 ? 16 : rows <= 32 ? 32 : rows <= 64 ? 64 : 128;
    const int S = B + 1;  // pooled-sequence slots
    std::vector<int32_t> lp(lens, lens + n_seq);
    if (B > rows) lp.push_back((int32_t)(B - rows));
    auto sets = prepare_pass(c, lp.data(), (int)lp.size(), B, S);
    Work& w = c->w;
    if ((long)S * total > w.pooled_cap || !w.dims) {
        CK(cudaStreamSynchronize(c->stream));
        dfree(c, w.pooled);
        w.pooled_cap = std::max((long)S * total, 4096L);
        w.pooled = (float*)dalloc(c, w.pooled_cap * 4);
        if (!w.dims) w.dims = (int*)dalloc(c, 64);
    }
    if (S > w.seq_meta_cap) {
        CK(cudaStreamSynchronize(c->stream));
        dfree(c, w.seq_meta);
        w.seq_meta_cap = std::max(S, 1024);
        w.seq_meta = (int*)dalloc(c, 2L * w.seq_meta_cap * 4);
    }
    const long need = pool_scratch_doubles(S, B, c->tc.emb);
    if (need > w.pool_scratch_cap) {
        CK(cudaStreamSynchronize(c->stream));
        dfree(c, w.pool_scratch);
        w.pool_scratch_cap = std::max(need, 1L << 20);
        w.pool_scratch = (double*)dalloc(c, w.pool_scratch_cap * 8);
    }
    // Metadata (the graph reads it from these fixed buffers): starts / lengths of S slots, dims, ids.
    std::vector<int> meta(2 * (size_t)S, 0);
    long r = 0;
    for (size_t s2 = 0; s2 < lp.size(); s2++) {
        meta[s2] = (int)r;
        meta[S + s2] = lp[s2];
        r += lp[s2];
    }
    int* seq_meta = w.seq_meta;
    CK(cudaMemcpyAsync(seq_meta, meta.data(), meta.size() * 4, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(w.dims, dims, n_dims * 4, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemsetAsync(w.ids, 0, (size_t)B * 4, c->stream));
    CK(cudaMemcpyAsync(w.ids, ids, rows * 4, ids_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, c->stream));
    auto body = [&]() {
        gather_pass(c, B);
        run_text(c, B, sets);
        KL(pool_rows(w.out, seq_meta, seq_meta + S, S, B, c->tc.emb, w.dims, n_dims, total, w.pooled, w.pool_scratch,
                     c->stream),
           "pool");
        g_launches.fetch_add(1, std::memory_order_relaxed);  // pool_rows is two launches
    };
    eg2_ctx::TextGraph* g = nullptr;
    for (auto& x : c->graphs)
        if (x.bucket == B && x.n_dims == n_dims && x.total == total) g = &x;
    if (g && g->gen == c->buf_gen) {
        CK(cudaGraphLaunch(g->exec, c->stream));
        g_launches.fetch_add(g->launches, std::memory_order_relaxed);
    } else {
        // Run the pass (this call's result, and it sets every kernel's attributes), then capture it on
        // a stream of the context's own; the capture itself runs nothing.
        body();
        if (!c->capture_stream) CK(cudaStreamCreateWithFlags(&c->capture_stream, cudaStreamNonBlocking));
        cudaStream_t saved = c->stream;
        c->stream = c->capture_stream;
        const long l0 = g_launches.load(std::memory_order_relaxed);
        cudaGraph_t graph = nullptr;
        CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
        try {
            body();
        } catch (...) {
            cudaStreamEndCapture(c->stream, &graph);
            if (graph) cudaGraphDestroy(graph);
            c->stream = saved;
            throw;
        }
        CK(cudaStreamEndCapture(c->stream, &graph));
        c->stream = saved;
        const long n_launch = g_launches.load(std::memory_order_relaxed) - l0;
        g_launches.fetch_sub(n_launch, std::memory_order_relaxed);  // captured, not run
        cudaGraphExec_t exec = nullptr;
        const cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        CK(e);
        if (!g) {
            c->graphs.push_back(eg2_ctx::TextGraph());
            g = &c->graphs.back();
        } else if (g->exec) {
            cudaGraphExecDestroy(g->exec);
        }
        g->bucket = B, g->n_dims = n_dims, g->total = total, g->gen = c->buf_gen, g->launches = n_launch, g->exec = exec;
    }
}

// One embedding pass of context c over `n_seq` sequences packed back to back (rows = sum(lens)), token
// ids at `ids` (host or device memory): pooled embeddings and their cuts in c->w.pooled [n_seq, total].
// Enqueued on c->stream; the caller reads c->bad_flag and the device status.
static void embed_pass(eg2_ctx* c, const uint32_t* ids, bool ids_on_device, const int32_t* lens, int n_seq, long rows,
                       const int32_t* dims, int n_dims, int total) {
    const bool graph_kind = (bf16_mode(c) && c->use_tc_attention) || c->precision == EG2_TF32;
    if (graph_kind && !c->profiling && rows <= 128 && !getenv("EG2_NO_GRAPHS")) {
        embed_graph(c, ids, lens, n_seq, rows, dims, n_dims, total, ids_on_device);
        return;
    }
    auto sets = prepare_pass(c, lens, n_seq, rows);
    Work& w = c->w;
    if ((long)n_seq * total > w.pooled_cap || !w.dims) {
        CK(cudaStreamSynchronize(c->stream));
        dfree(c, w.pooled);
        w.pooled_cap = std::max((long)n_seq * total, 4096L);
        w.pooled = (float*)dalloc(c, w.pooled_cap * 4);
        if (!w.dims) w.dims = (int*)dalloc(c, 64);
    }
    std::vector<int> st(n_seq), ln(n_seq);
    long r = 0;
    for (int s = 0; s < n_seq; s++) {
        st[s] = (int)r;
        ln[s] = lens[s];
        r += lens[s];
    }
    // Per-sequence start / length for the pool kernel.
    if (n_seq > w.seq_meta_cap) {
        CK(cudaStreamSynchronize(c->stream));
        dfree(c, w.seq_meta);
        w.seq_meta_cap = std::max(n_seq, 1024);
        w.seq_meta = (int*)dalloc(c, 2L * w.seq_meta_cap * 4);
    }
    int* seq_meta = w.seq_meta;
    CK(cudaMemcpyAsync(seq_meta, st.data(), n_seq * 4, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(seq_meta + n_seq, ln.data(), n_seq * 4, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(w.dims, dims, n_dims * 4, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(w.ids, ids, rows * 4, ids_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, c->stream));
    gather_pass(c, rows);
    run_text(c, rows, sets);
    int max_len = 0;
    for (int s2 = 0; s2 < n_seq; s2++) max_len = std::max(max_len, (int)lens[s2]);
    const long need = pool_scratch_doubles(n_seq, max_len, c->tc.emb);
    if (need > w.pool_scratch_cap) {
        CK(cudaStreamSynchronize(c->stream));
        dfree(c, w.pool_scratch);
        w.pool_scratch_cap = std::max(need, 1L << 20);
        w.pool_scratch = (double*)dalloc(c, w.pool_scratch_cap * 8);
    }
    KL(pool_rows(w.out, seq_meta, seq_meta + n_seq, n_seq, max_len, c->tc.emb, w.dims, n_dims, total, w.pooled,
                 w.pool_scratch, c->stream),
       "pool");
    g_launches.fetch_add(1, std::memory_order_relaxed);  // pool_rows is two launches
    mark(c, "pool");
}

static int embed_impl(eg2_ctx* c, const uint32_t* ids, const int32_t* lens, int n_seq, const int32_t* dims, int n_dims,
                      float* out, void* stream, bool device_ptrs) {
    return guarded(c, [&] {
        cudaStream_t saved = c->stream;
        if (stream) c->stream = (cudaStream_t)stream;
        struct Restore {
            eg2_ctx* c;
            cudaStream_t s;
            ~Restore() { c->stream = s; }
        } restore{c, saved};
        const long rows = check_lens(lens, n_seq);
        if (rows == 0) return;
        if (!ids || !out || !dims || n_dims <= 0 || n_dims > 16) fail(EG2_ERR_INVALID, "bad arguments");
        int total = 0;
        for (int d = 0; d < n_dims; d++) {
            if (dims[d] <= 0 || dims[d] > c->tc.emb) fail(EG2_ERR_INVALID, "truncate_dim %d out of range 1..=%d", dims[d], c->tc.emb);
            total += dims[d];
        }
        if (!device_ptrs)
            for (long i = 0; i < rows; i++)
                if ((int64_t)ids[i] >= c->tc.vocab) fail(EG2_ERR_INVALID, "token id %u out of range", ids[i]);
        mark(c, "call");  // profiling: the interval up to the first kernel is the host's set-up of the pass
        const auto plan = call_plan(c, lens, n_seq);
        CK(cudaMemsetAsync(c->bad_flag, 0, 4, c->stream));
        if (c->precise) CK(cudaMemsetAsync(c->precise->bad_flag, 0, 4, c->stream));
        const float* result = nullptr;
        if (plan.size() == 1) {
            eg2_ctx* x = plan[0].precise ? c->precise : c;
            embed_pass(x, ids, device_ptrs, lens, n_seq, rows, dims, n_dims, total);
            result = x->w.pooled;
        } else {
            // Several passes: each pass's ids are gathered into one contiguous buffer, its pooled rows
            // scattered into the call's result buffer, which reaches `out` once every pass succeeded.
            long max_pass = 0;
            for (const Pass& p : plan) max_pass = std::max(max_pass, p.rows);
            ensure_stage(c, device_ptrs ? max_pass : 0, (long)n_seq * total);
            const auto seq_row0 = row_offsets(lens, n_seq);
            for (const Pass& p : plan) {
                eg2_ctx* x = p.precise ? c->precise : c;
                const auto runs = pass_runs(p, seq_row0, lens);
                std::vector<int32_t> plens;
                for (int s : p.seqs) plens.push_back(lens[s]);
                std::vector<uint32_t> hids;
                const uint32_t* pids;
                if (device_ptrs) {
                    for (const Run& r : runs)
                        CK(cudaMemcpyAsync(c->stage_ids + r.prow0, ids + r.row0, r.rows * 4, cudaMemcpyDeviceToDevice,
                                           c->stream));
                    pids = c->stage_ids;
                } else {
                    hids.resize(p.rows);
                    for (const Run& r : runs) memcpy(hids.data() + r.prow0, ids + r.row0, r.rows * 4);
                    pids = hids.data();
                }
                // (A host `pids` is pageable: its copy completes before embed_pass returns.)
                embed_pass(x, pids, device_ptrs, plens.data(), (int)plens.size(), p.rows, dims, n_dims, total);
                for (const Run& r : runs)
                    CK(cudaMemcpyAsync(c->stage_out + (long)r.seq0 * total, x->w.pooled + (long)r.pseq0 * total,
                                       (long)r.nseq * total * 4, cudaMemcpyDeviceToDevice, c->stream));
            }
            result = c->stage_out;
        }
        int bad = 0, bad_precise = 0;
        CK(cudaMemcpyAsync(&bad, c->bad_flag, 4, cudaMemcpyDeviceToHost, c->stream));
        if (c->precise) CK(cudaMemcpyAsync(&bad_precise, c->precise->bad_flag, 4, cudaMemcpyDeviceToHost, c->stream));
        check_device_status(c);
        if (bad || bad_precise) fail(EG2_ERR_INVALID, "token id out of range");
        CK(cudaMemcpyAsync(out, result, (size_t)n_seq * total * 4, device_ptrs ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost,
                           c->stream));
        mark(c, "checks + output");
        CK(cudaStreamSynchronize(c->stream));
        collect_marks(c);
    });
}

int eg2_embed_packed(eg2_ctx* c, const uint32_t* ids, const int32_t* lens, int n_seq, const int32_t* dims, int n_dims,
                     float* out) {
    return embed_impl(c, ids, lens, n_seq, dims, n_dims, out, nullptr, false);
}
int eg2_embed_packed_device(eg2_ctx* c, const uint32_t* ids, const int32_t* lens, int n_seq, const int32_t* dims,
                            int n_dims, float* out, void* stream) {
    return embed_impl(c, ids, lens, n_seq, dims, n_dims, out, stream, true);
}

int eg2_plan_passes(const int32_t* lens, int n_seq, int64_t max_rows, int precise_max, int32_t* pass_of_seq,
                    int32_t* pass_precise) {
    if (n_seq < 0 || (n_seq > 0 && (!lens || !pass_of_seq)) || max_rows <= 0 || precise_max < 0) return EG2_ERR_INVALID;
    for (int s = 0; s < n_seq; s++)
        if (lens[s] <= 0) return EG2_ERR_INVALID;
    const auto plan = plan_passes(lens, n_seq, (long)max_rows, precise_max);
    for (size_t p = 0; p < plan.size(); p++) {
        for (int s : plan[p].seqs) pass_of_seq[s] = (int32_t)p;
        if (pass_precise) pass_precise[p] = plan[p].precise ? 1 : 0;
    }
    return (int)plan.size();
}

int eg2_pass_policy(const eg2_ctx* c, int64_t* max_rows, int* precise_max) {
    if (!c) return EG2_ERR_INVALID;
    if (max_rows) *max_rows = c->pass_rows;
    if (precise_max) *precise_max = (c->precise && c->precision == EG2_BF16) ? c->precise_max : 0;
    return EG2_OK;
}

// The vision tower over n_img images of one patch grid (gh x gw, positions pos_xy shared), stacked
// image after image into one device pass.
static int vision_impl(eg2_ctx* c, const float* patches, const int32_t* pos_xy, int n_img, int gh, int gw,
                       float* out_pooled, float* out_soft) {
    return guarded(c, [&] {
        VisionCfg& vc = c->vc;
        if (!vc.present) fail(EG2_ERR_INVALID, "the checkpoint has no vision tower");
        const int k = vc.pool;
        const long per = (long)gh * gw;
        if (gh <= 0 || gw <= 0 || gh % k || gw % k)
            fail(EG2_ERR_INVALID, "patch grid %dx%d is empty or not divisible by the pooling kernel %d", gh, gw, k);
        if (n_img <= 0 || per * n_img > (1L << 26)) fail(EG2_ERR_INVALID, "bad image count %d", n_img);
        if (!patches || !pos_xy) fail(EG2_ERR_INVALID, "null buffer");
        for (long t = 0; t < per; t++)
            if (pos_xy[2 * t] < 0 || pos_xy[2 * t] >= vc.pos_size || pos_xy[2 * t + 1] < 0 || pos_xy[2 * t + 1] >= vc.pos_size)
                fail(EG2_ERR_INVALID, "patch position outside the %d-entry position table", vc.pos_size);
        const long n = per * n_img;
        const int h = vc.hidden, ff = vc.inter, nh = vc.nh, nkv = vc.nkv, hd = vc.hd, pd = 3 * vc.patch * vc.patch;
        const size_t as = act_size(c);
        if (n > c->vcap) {
            CK(cudaStreamSynchronize(c->stream));
            void** bufs[] = {(void**)&c->v_hidden, (void**)&c->v_pooled, (void**)&c->v_cs, (void**)&c->v_sn, (void**)&c->v_soft,
                             (void**)&c->v_inv,
                             &c->v_x, &c->v_t, &c->v_qkv, &c->v_q, &c->v_k, &c->v_v, &c->v_a, &c->v_o, &c->v_gate, &c->v_gu,
                             (void**)&c->v_pos, (void**)&c->v_seq_start, (void**)&c->v_seq_len, (void**)&c->v_tiles};
            for (void** b : bufs) {
                dfree(c, *b);
                *b = nullptr;
            }
            c->v_tiles_cap = 0;
            const long cap = ((n + 1023) / 1024) * 1024;
            const size_t per_row = (size_t)h * 4 * 3 + (size_t)c->tc.hidden * 4 + (size_t)hd * 4 + (size_t)pd * 4 +
                                   (size_t)std::max(h, pd) * as + (size_t)(nh + 2 * nkv) * hd * (4 + as) +
                                   (size_t)nh * hd * as + (size_t)ff * as + (c->precision == EG2_F32 ? 2 * (size_t)ff * 4 : 0) + 16;
            ensure_fits(per_row * cap, "the vision workspace", n);
            c->v_hidden = (float*)dalloc(c, cap * h * 4);
            c->v_pooled = (float*)dalloc(c, cap * h * 4);
            c->v_soft = (float*)dalloc(c, cap * c->tc.hidden * 4);
            c->v_cs = (float*)dalloc(c, cap * (hd / 2) * 4);
            c->v_sn = (float*)dalloc(c, cap * (hd / 2) * 4);
            c->v_inv = (float*)dalloc(c, 4 * hd);
            c->v_x = dalloc(c, cap * pd * 4);
            c->v_t = dalloc(c, cap * std::max(h, pd) * as);
            c->v_qkv = dalloc(c, cap * (nh + 2 * nkv) * hd * 4);
            c->v_q = dalloc(c, cap * nh * hd * as);
            c->v_k = dalloc(c, cap * nkv * hd * as);
            c->v_v = dalloc(c, cap * nkv * hd * as);
            c->v_a = dalloc(c, cap * nh * hd * as);
            c->v_o = dalloc(c, cap * h * 4);
            c->v_gate = dalloc(c, cap * ff * as);
            c->v_gu = c->precision == EG2_F32 ? dalloc(c, cap * 2L * ff * 4) : nullptr;
            c->v_pos = (int*)dalloc(c, cap * 2 * 4);
            c->v_seq_start = (int*)dalloc(c, cap * 4);
            c->v_seq_len = (int*)dalloc(c, cap * 4);
            c->v_tiles_cap = 0;
            c->v_pos_host.clear();
            c->vcap = cap;
        }
        // Query tiles: 256 patches of one image each, so their count depends on the image count as well
        // as on the rows.
        const int n_tiles = (int)(n_img * ((per + 255) / 256));
        if (n_tiles > c->v_tiles_cap) {
            CK(cudaStreamSynchronize(c->stream));
            dfree(c, c->v_tiles);
            c->v_tiles_cap = std::max<long>(n_tiles, c->vcap / 256 + 1);
            c->v_tiles = (AttnTile*)dalloc(c, c->v_tiles_cap * sizeof(AttnTile));
            c->v_pos_host.clear();  // the tile list is rebuilt with the tables below
        }
        // Position-dependent tables, rebuilt only when the positions (or the image count) differ from the
        // previous call's (images of one size share them).
        if (c->v_pos_host.size() != (size_t)(2 * per + 1) || c->v_pos_host[2 * per] != n_img ||
            std::memcmp(c->v_pos_host.data(), pos_xy, (size_t)per * 2 * sizeof(int32_t)) != 0) {
            // Axial RoPE tables [n, hd / 2]: x angles in the first hd / 4 entries, y in the next (src/vision.rs:114-136).
            std::vector<float> inv = rope_inv_freq(vc.theta, hd / 2);
            const int q4 = hd / 4;
            // One image's tables, then copies for the other images of the call.
            const size_t rw = (size_t)(hd / 2);
            std::vector<float> cs((size_t)n * rw), sn((size_t)n * rw);
            std::vector<int32_t> pos((size_t)n * 2);
            for (long t = 0; t < per; t++)
                for (int axis = 0; axis < 2; axis++)
                    for (int i = 0; i < q4; i++) {
                        const float f = (float)pos_xy[2 * t + axis] * inv[i];
                        const int col = axis * q4 + i;
                        cs[(size_t)t * rw + col] = cosf(f);
                        sn[(size_t)t * rw + col] = sinf(f);
                    }
            for (int im = 0; im < n_img; im++) {
                if (im > 0) {
                    std::copy(cs.begin(), cs.begin() + per * rw, cs.begin() + im * per * rw);
                    std::copy(sn.begin(), sn.begin() + per * rw, sn.begin() + im * per * rw);
                }
                std::copy(pos_xy, pos_xy + 2 * per, pos.begin() + (size_t)im * per * 2);
            }
            // Each image is one sequence: row metadata for the CUDA-core attention, 256-token tiles for
            // the tensor-core one.
            std::vector<int> starts(n), lens_v(n, (int)per);
            std::vector<AttnTile> tiles;
            for (int im = 0; im < n_img; im++) {
                for (long t = 0; t < per; t++) starts[im * per + t] = (int)(im * per);
                for (int q0 = 0; q0 < per; q0 += 256) tiles.push_back(AttnTile{(int)(im * per), (int)per, q0});
            }
            CK(cudaMemcpyAsync(c->v_inv, inv.data(), inv.size() * 4, cudaMemcpyHostToDevice, c->stream));
            CK(cudaMemcpyAsync(c->v_cs, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, c->stream));
            CK(cudaMemcpyAsync(c->v_sn, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice, c->stream));
            CK(cudaMemcpyAsync(c->v_pos, pos.data(), pos.size() * 4, cudaMemcpyHostToDevice, c->stream));
            CK(cudaMemcpyAsync(c->v_seq_start, starts.data(), n * 4, cudaMemcpyHostToDevice, c->stream));
            CK(cudaMemcpyAsync(c->v_seq_len, lens_v.data(), n * 4, cudaMemcpyHostToDevice, c->stream));
            CK(cudaMemcpyAsync(c->v_tiles, tiles.data(), tiles.size() * sizeof(AttnTile), cudaMemcpyHostToDevice, c->stream));
            // The host vectors die at the end of this block.
            CK(cudaStreamSynchronize(c->stream));
            c->v_pos_host.assign(pos_xy, pos_xy + 2 * per);
            c->v_pos_host.push_back(n_img);
        }
        CK(cudaMemcpyAsync(c->v_x, patches, n * pd * 4, cudaMemcpyHostToDevice, c->stream));
        // 2 (x - 0.5) into the GEMM input buffer in the storage type.
        if (bf16_mode(c))
            KL(cast_rows<bf16_t>((const float*)c->v_x, (bf16_t*)c->v_t, n * pd, 2.f, -0.5f, c->stream), "cast");
        else
            KL(cast_rows<float>((const float*)c->v_x, (float*)c->v_t, n * pd, 2.f, -0.5f, c->stream), "cast");
        if (bf16_mode(c))
            enqueue_vision<bf16_t>(c, n, gh, gw, n_img, n_tiles);
        else
            enqueue_vision<float>(c, n, gh, gw, n_img, n_tiles);
        const long no = (long)n_img * (gh / k) * (gw / k);
        check_device_status(c);
        if (out_pooled) CK(cudaMemcpyAsync(out_pooled, c->v_pooled, no * h * 4, cudaMemcpyDeviceToHost, c->stream));
        if (out_soft) CK(cudaMemcpyAsync(out_soft, c->v_soft, no * c->tc.hidden * 4, cudaMemcpyDeviceToHost, c->stream));
        CK(cudaStreamSynchronize(c->stream));
        collect_marks(c);
    });
}

int eg2_vision_encode(eg2_ctx* c, const float* patches, const int32_t* pos_xy, int gh, int gw, float* out_pooled,
                      float* out_soft) {
    return vision_impl(c, patches, pos_xy, 1, gh, gw, out_pooled, out_soft);
}

int eg2_vision_encode_batch(eg2_ctx* c, const float* patches, const int32_t* pos_xy, int n_images, int gh, int gw,
                            float* out_pooled, float* out_soft) {
    return vision_impl(c, patches, pos_xy, n_images, gh, gw, out_pooled, out_soft);
}

int eg2_profile(eg2_ctx* c, int enable) {
    return guarded(c, [&] {
        c->profiling = enable != 0;
        c->prof.clear();
    });
}

int eg2_profile_read(eg2_ctx* c, char* buf, int cap) {
    return guarded(c, [&] {
        std::string s = "{";
        bool first = true;
        for (auto& kv : c->prof) {
            char item[256];
            snprintf(item, sizeof item, "%s\"%s\": [%.6f, %ld]", first ? "" : ", ", kv.first.c_str(), kv.second.first,
                     kv.second.second);
            s += item;
            first = false;
        }
        s += "}";
        if (!buf || cap <= (int)s.size()) fail(EG2_ERR_INVALID, "buffer too small (%zu bytes needed)", s.size() + 1);
        memcpy(buf, s.c_str(), s.size() + 1);
    });
}

int eg2_gemm(int kind, const void* A, int64_t lda, const void* W, int64_t ldw, void* C, int64_t ldc, int M, int N, int K,
             int out_f32, void* stream) {
    if (!A || !W || !C || M < 0 || N <= 0 || K <= 0) return EG2_ERR_INVALID;
    cudaStream_t s = (cudaStream_t)stream;
    int rc;
    if (kind == EG2_F32) {
        rc = gemm_f32((const float*)A, lda, (const float*)W, ldw, (float*)C, ldc, M, N, K, 1.f, s);
    } else if (kind == EG2_BF16 || kind == EG2_TF32) {
        GemmEpilogue e;
        e.mode = EPI_STORE;
        e.out_f32 = (kind == EG2_TF32 || out_f32) ? 1 : 0;
        e.out = C;
        e.ldo = ldc;
        rc = gemm_tc(kind == EG2_BF16 ? GEMM_BF16 : GEMM_TF32, A, lda, W, ldw, M, N, K, e, s);
    } else {
        return EG2_ERR_INVALID;
    }
    if (rc == -1) return EG2_ERR_INVALID;
    return rc ? EG2_ERR_CUDA : EG2_OK;
}

int eg2_attention(int kind, const void* q, const void* k, const void* v, void* out, const int32_t* lens, int n_seq, int nh,
                  int nkv, int hd, int window, void* stream) {
    if (!q || !k || !v || !out || !lens || n_seq <= 0 || nh <= 0 || nkv <= 0 || nh % nkv) return EG2_ERR_INVALID;
    cudaStream_t s = (cudaStream_t)stream;
    long rows = 0;
    for (int i = 0; i < n_seq; i++) {
        if (lens[i] <= 0) return EG2_ERR_INVALID;
        rows += lens[i];
    }
    std::vector<int> st(rows), ln(rows);
    std::vector<AttnTile> tiles;
    long r = 0;
    const int tq = kind == EG2_BF16 ? attention_tc_tile_tokens(nh, nkv, hd) : 0;
    if (kind == EG2_BF16 && tq <= 0) return EG2_ERR_INVALID;
    for (int i = 0; i < n_seq; i++) {
        for (int j = 0; j < lens[i]; j++) {
            st[r + j] = (int)r;
            ln[r + j] = lens[i];
        }
        if (tq > 0)
            for (int q0 = 0; q0 < lens[i]; q0 += tq) tiles.push_back(AttnTile{(int)r, lens[i], q0});
        r += lens[i];
    }
    int* meta = nullptr;
    AttnTile* dt = nullptr;
    if (cudaMalloc(&meta, 2 * rows * 4) != cudaSuccess) return EG2_ERR_OOM;
    if (!tiles.empty() && cudaMalloc(&dt, tiles.size() * sizeof(AttnTile)) != cudaSuccess) {
        cudaFree(meta);
        return EG2_ERR_OOM;
    }
    cudaMemcpyAsync(meta, st.data(), rows * 4, cudaMemcpyHostToDevice, s);
    cudaMemcpyAsync(meta + rows, ln.data(), rows * 4, cudaMemcpyHostToDevice, s);
    if (dt) cudaMemcpyAsync(dt, tiles.data(), tiles.size() * sizeof(AttnTile), cudaMemcpyHostToDevice, s);
    int rc;
    if (kind == EG2_F32)
        rc = attention_simt<float>((const float*)q, (const float*)k, (const float*)v, (float*)out, meta, meta + rows, rows, nh,
                                   nkv, hd, window, s);
    else if (kind == EG2_BF16)
        rc = attention_tc((const bf16_t*)q, (const bf16_t*)k, (const bf16_t*)v, (bf16_t*)out, rows, dt, (int)tiles.size(),
                          nh, nkv, hd, window, s);
    else
        rc = -1;
    cudaStreamSynchronize(s);
    cudaFree(meta);
    if (dt) cudaFree(dt);
    if (rc == -1) return EG2_ERR_INVALID;
    if (rc) return EG2_ERR_CUDA;
    int stv = 0;
    cudaMemcpyFromSymbol(&stv, eg2_dev_status, sizeof(int));
    return stv ? EG2_ERR_TIMEOUT : EG2_OK;
}

int eg2_attention_noalloc(const void* q, const void* k, const void* v, void* out, const int32_t* lens, int n_seq, int nh,
                          int nkv, int hd, int window, void* stream) {
    const int rc = attention_noalloc((const bf16_t*)q, (const bf16_t*)k, (const bf16_t*)v, (bf16_t*)out, lens, n_seq, nh,
                                     nkv, hd, window, (cudaStream_t)stream);
    if (rc == -1) return EG2_ERR_INVALID;
    if (rc) return EG2_ERR_CUDA;
    g_launches.fetch_add(2, std::memory_order_relaxed);
    return EG2_OK;
}

long long eg2_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int eg2_device_status(void) {
    int st = 0;
    cudaMemcpyFromSymbol(&st, eg2_dev_status, sizeof(int));
    return st;
}
void eg2_device_status_reset(void) {
    int zero = 0;
    cudaMemcpyToSymbol(eg2_dev_status, &zero, sizeof(int));
}

int eg2_wait_timeout_probe(int device, unsigned int limit_us, int* device_status) {
    if (!device_status || limit_us == 0 || limit_us > 2000000u) return EG2_ERR_INVALID;
    if (cudaSetDevice(device) != cudaSuccess) return EG2_ERR_CUDA;
    eg2_device_status_reset();
    if (wait_timeout_probe((unsigned long long)limit_us * 1000ull, nullptr)) return EG2_ERR_CUDA;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (cudaDeviceSynchronize() != cudaSuccess) return EG2_ERR_CUDA;
    *device_status = eg2_device_status();
    eg2_device_status_reset();
    return EG2_OK;
}

}  // extern "C"

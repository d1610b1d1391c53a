// Allocation-free variant of the attention entry point (eg2_attention_noalloc in include/eg2.h).
//
// eg2_attention keeps its per-call scratch -- the sequence lengths and the list of query tiles the
// tensor-core kernel walks -- in device buffers it allocates and frees on every call. Some callers
// cannot allow that: a serving engine that reserves all device memory for its own pool up front (a
// cudaMalloc behind its back can fail or fragment that pool), or a latency-critical path where the
// implicit device synchronisation of cudaMalloc / cudaFree would stall work on other streams. For
// them this variant keeps the scratch in a file-scope device array of fixed size that every GPU
// loading the library holds until the process exits, builds the tile list there with a small
// kernel, and calls no allocating routine.
//
// Limits: at most EG2_NOALLOC_MAX_SEQ sequences and EG2_NOALLOC_MAX_TILES query tiles per call
// (a tile is up to 128 query tokens of one sequence for 4 query heads over 2 K/V heads of 256, 64 for
// 4 over 1 of 512, 256 for head 64), i.e. 4 M to 16 M rows; larger calls are rejected.
// All calls share the one array and leave their contents in it: two calls that overlap on the GPU
// (different streams, or different host threads, with no ordering between them) race on it.
// The call is asynchronous: a bounded device wait that ran out is reported through the device
// status word (eg2_device_status), which the caller reads after synchronising the stream.
#include "common.cuh"
#include "kernels.h"

#include <cstddef>
#include <mutex>

namespace eg2 {

constexpr int EG2_NOALLOC_MAX_SEQ = 65536;
constexpr int EG2_NOALLOC_MAX_TILES = 65536;

struct NoAllocScratch {
    int lens[EG2_NOALLOC_MAX_SEQ];
    AttnTile tiles[EG2_NOALLOC_MAX_TILES];
};

// 1 MiB per device, for the lifetime of the process.
static __device__ __align__(256) NoAllocScratch g_noalloc_scratch;

// One block: exclusive scans of the row offsets and of the tiles per sequence, then every tile.
// Writes exactly n_tiles entries (the host computed n_tiles from the same lengths), so nothing from
// an earlier call is read.
__global__ void build_tiles_kernel(NoAllocScratch* sc, int n_seq, int tq) {
    __shared__ long long row_base[1024];
    __shared__ int tile_base[1024];
    const int per = (n_seq + blockDim.x - 1) / blockDim.x;
    const int s0 = threadIdx.x * per, s1 = min(n_seq, s0 + per);
    long long rows = 0;
    int tiles = 0;
    for (int s = s0; s < s1; s++) {
        rows += sc->lens[s];
        tiles += (sc->lens[s] + tq - 1) / tq;
    }
    row_base[threadIdx.x] = rows;
    tile_base[threadIdx.x] = tiles;
    __syncthreads();
    if (threadIdx.x == 0) {
        long long r = 0;
        int t = 0;
        for (int i = 0; i < (int)blockDim.x; i++) {
            const long long rr = row_base[i];
            const int tt = tile_base[i];
            row_base[i] = r;
            tile_base[i] = t;
            r += rr;
            t += tt;
        }
    }
    __syncthreads();
    long long row0 = row_base[threadIdx.x];
    int t = tile_base[threadIdx.x];
    for (int s = s0; s < s1; s++) {
        const int len = sc->lens[s];
        for (int q0 = 0; q0 < len; q0 += tq) sc->tiles[t++] = AttnTile{(int)row0, len, q0};
        row0 += len;
    }
}

static NoAllocScratch* scratch_address() {
    // The device address of the array, looked up once per device with that device current. In host
    // code `g_noalloc_scratch` names a host-side stand-in, never the device memory.
    static std::mutex mu;
    static NoAllocScratch* addr[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        addr[dev] = static_cast<NoAllocScratch*>(p);
    }
    return addr[dev];
}

int attention_noalloc(const bf16_t* q, const bf16_t* k, const bf16_t* v, bf16_t* out, const int32_t* lens, int n_seq,
                      int nh, int nkv, int hd, int window, cudaStream_t s) {
    // Every argument is checked on the host before anything is copied or launched.
    if (!q || !k || !v || !out || !lens || n_seq <= 0 || n_seq > EG2_NOALLOC_MAX_SEQ) return -1;
    if (nh <= 0 || nkv <= 0 || nh % nkv) return -1;
    const int tq = attention_tc_tile_tokens(nh, nkv, hd);
    if (tq <= 0) return -1;
    long rows = 0, n_tiles = 0;
    for (int i = 0; i < n_seq; i++) {
        if (lens[i] <= 0) return -1;
        rows += lens[i];
        n_tiles += (lens[i] + tq - 1) / tq;
    }
    if (n_tiles > EG2_NOALLOC_MAX_TILES || rows > (1L << 30)) return -1;
    NoAllocScratch* sc = scratch_address();
    if (!sc) return -3;
    // The lengths go into the array (from the caller's host memory), then the tile list is built there.
    // From pageable host memory the copy reads `lens` before cudaMemcpyAsync returns; from page-locked
    // memory it is asynchronous and reads `lens` when the stream reaches it.
    // (Addresses inside the device array are formed by offset arithmetic; nothing is dereferenced here.)
    int* d_lens = reinterpret_cast<int*>(reinterpret_cast<char*>(sc) + offsetof(NoAllocScratch, lens));
    AttnTile* d_tiles = reinterpret_cast<AttnTile*>(reinterpret_cast<char*>(sc) + offsetof(NoAllocScratch, tiles));
    if (cudaMemcpyAsync(d_lens, lens, (size_t)n_seq * sizeof(int), cudaMemcpyHostToDevice, s) != cudaSuccess) return -3;
    build_tiles_kernel<<<1, 1024, 0, s>>>(sc, n_seq, tq);
    if (cudaGetLastError() != cudaSuccess) return -3;
    return attention_tc(q, k, v, out, rows, d_tiles, (int)n_tiles, nh, nkv, hd, window, s);
}

}  // namespace eg2

// Shared device helpers for the sm_100a kernels: bf16 conversion, mbarriers with bounded waits,
// TMA tile loads, tcgen05 (TMEM allocation, MMA issue, commit, TMEM loads) and UMMA descriptors.
//
// Every wait on an mbarrier is bounded by wall time (%globaltimer). A wait that runs out records
// an error code in eg2_dev_status (read back by the host after the launch) and returns false, so
// a kernel with a broken pipeline ends with an error status instead of hanging the GPU.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

typedef uint16_t bf16_t;

#define EG2_DEV __device__ __forceinline__

// Device-side status word: 0 = fine, otherwise the first error code recorded by any kernel.
__device__ int eg2_dev_status = 0;

enum Eg2DevError : int {
    EG2_DEV_OK = 0,
    EG2_DEV_TIMEOUT_GEMM = 1,
    EG2_DEV_TIMEOUT_ATTN = 2,
    EG2_DEV_BAD_ARGS = 3,
    EG2_DEV_TIMEOUT_PROBE = 4,  // the failure-detection probe's wait ran out (as designed)
};

// Upper bound of any single wait: 2 s. A healthy pipeline waits microseconds.
#define EG2_WAIT_LIMIT_NS 2000000000ull

EG2_DEV void eg2_record_error(int code) { atomicCAS(&eg2_dev_status, 0, code); }

// ---------------------------------------------------------------------------------------------
// bf16
// ---------------------------------------------------------------------------------------------
EG2_DEV float bf16_to_f32(bf16_t b) { return __uint_as_float(((uint32_t)b) << 16); }
EG2_DEV bf16_t f32_to_bf16(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }
EG2_DEV uint32_t pack_bf16x2(float lo, float hi) {
    return (uint32_t)f32_to_bf16(lo) | ((uint32_t)f32_to_bf16(hi) << 16);
}

// 2^x on the MUFU unit (flush-to-zero; ex2(-inf) = +0).
EG2_DEV float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// Two floats to packed bf16 (round to nearest even) in one cvt: lo in bits 0-15.
EG2_DEV uint32_t bf16x2_bits(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// sin and cos of an angle of moderate size (|a| < 2^12 * 2 pi): Cody-Waite reduction by 2 pi
// (6.28125 has 8 significant bits, so k * 6.28125 is exact for |k| < 2^15), then the MUFU
// approximations, which are accurate to ~4e-7 absolute on [-pi, pi]. k = the nearest integer to
// a / (2 pi), ties to even, by adding and subtracting 1.5 * 2^23 (exact for |a / (2 pi)| < 2^22; the
// same value as rintf, on the FMA pipe instead of a rounding instruction).
EG2_DEV void sincos_reduced(float a, float& s, float& c) {
    const float k = __fsub_rn(__fadd_rn(a * 0.15915494309189535f, 12582912.f), 12582912.f);
    float r = fmaf(-k, 6.28125f, a);
    r = fmaf(-k, 1.9353071795864769e-3f, r);
    s = __sinf(r);
    c = __cosf(r);
}

// GELU with the tanh approximation (the reference's gelu_tanh, constants as written there).
EG2_DEV float gelu_tanh_f(float x) {
    const float beta = 0.79788456f, kappa = 0.044715f;
    float inner = beta * (x + kappa * x * x * x);
    return 0.5f * x * (1.f + tanhf(inner));
}

// Load / store one element of f32 or bf16 storage as f32.
template <typename T>
EG2_DEV float ldf(const T* p, long i);
template <>
EG2_DEV float ldf<float>(const float* p, long i) {
    return p[i];
}
template <>
EG2_DEV float ldf<bf16_t>(const bf16_t* p, long i) {
    return bf16_to_f32(p[i]);
}
template <typename T>
EG2_DEV void stf(T* p, long i, float v);
template <>
EG2_DEV void stf<float>(float* p, long i, float v) {
    p[i] = v;
}
template <>
EG2_DEV void stf<bf16_t>(bf16_t* p, long i, float v) {
    p[i] = f32_to_bf16(v);
}

EG2_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

EG2_DEV uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

EG2_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// ---------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------
EG2_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
EG2_DEV void fence_mbarrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
EG2_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

EG2_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}
EG2_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
EG2_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase with the given parity to complete. Returns false (and records
// `code`) if it does not complete within `limit_ns`, or if `abort` is already set.
EG2_DEV bool mbar_wait_limit(uint64_t* bar, uint32_t parity, int code, volatile int* abort, uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 255u) {
            if (abort && *abort) return false;
            // Another CTA already gave up: stop waiting too, so a broken launch ends in ~2 s.
            if (*(volatile int*)&eg2_dev_status != 0) {
                if (abort) *abort = 1;
                return false;
            }
            if (globaltimer_ns() - t0 > limit_ns) {
                eg2_record_error(code);
                if (abort) *abort = 1;
                return false;
            }
        }
    }
}
EG2_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, int code, volatile int* abort) {
    return mbar_wait_limit(bar, parity, code, abort, EG2_WAIT_LIMIT_NS);
}
// Exit path: waits (at most limit_ns, whatever the error state) for a copy this CTA issued to land,
// so no TMA write reaches shared memory after the CTA has ended.
EG2_DEV void mbar_drain(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return;
        if ((it & 255u) == 255u && globaltimer_ns() - t0 > limit_ns) return;
    }
}

// ---------------------------------------------------------------------------------------------
// Thread-block clusters: distributed shared memory between the CTAs of a cluster
// ---------------------------------------------------------------------------------------------
EG2_DEV uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// All threads of every CTA of the cluster; orders earlier shared-memory writes (and mbarrier
// initialisation) before later accesses from the other CTAs.
EG2_DEV void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The shared::cluster address of the variable at `local` (this CTA's shared memory) in CTA `rank`.
EG2_DEV uint32_t mapa_shared(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}
// Arrive on an mbarrier of another CTA of the cluster (default release.cta semantics: enough when
// the data it guards is ordered otherwise, e.g. TMEM through tcgen05 fences; a cluster-scope release
// here costs ~1,000 cycles per arrive).
EG2_DEV void mbar_arrive_remote(uint32_t remote_bar) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(remote_bar) : "memory");
}
// Store a 32-bit value into another CTA's shared memory and count its 4 bytes as completed
// transactions on that CTA's mbarrier `remote_bar` (both shared::cluster addresses of the same CTA).
// A thread that sees the barrier's phase complete also sees the value.
EG2_DEV void st_async_f32(uint32_t remote_addr, float v, uint32_t remote_bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(remote_addr), "f"(v),
                 "r"(remote_bar)
                 : "memory");
}
// Bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned) from this CTA's shared
// memory at `src` to shared::cluster address `dst` of another CTA, completing the bytes on that
// CTA's mbarrier `remote_bar`. Writer threads make their stores to `src` visible to the copy with
// fence.proxy.async before it is issued; `src` may be rewritten once the destination barrier says
// the bytes have landed.
EG2_DEV void bulk_copy_to_peer(uint32_t dst, uint32_t src, uint32_t bytes, uint32_t remote_bar) {
    asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "r"(src), "r"(bytes), "r"(remote_bar)
                 : "memory");
}
// ---------------------------------------------------------------------------------------------
// TMA (tiled tensor loads into this CTA's own shared memory)
// ---------------------------------------------------------------------------------------------
EG2_DEV void tma_prefetch_desc(const CUtensorMap* m) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
// Bulk prefetch of `bytes` (multiple of 16, 16-byte aligned address) of global memory into L2.
// TMA store of a tile from this CTA's shared memory (box and swizzle from the tensor map); rows and
// columns outside the tensor are not written. Completion is tracked by bulk async-groups of the
// issuing thread: commit after issuing, then wait_group[.read] on the same thread.
EG2_DEV void tma_store_2d(const CUtensorMap* m, const void* src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(m)),
                 "r"(smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
}
EG2_DEV void tma_store_3d(const CUtensorMap* m, const void* src, int x, int y, int z) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(m)),
                 "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
                 : "memory");
}
EG2_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Programmatic dependent launch: let the next kernel on the stream start launching (its CTAs run
// their prologue up to grid_dep_wait), and wait until the previous kernel has completed and its
// writes are visible (returns at once when this kernel was not launched as a dependent).
EG2_DEV void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
EG2_DEV void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// 32-byte store (p 32-byte aligned): a warp of these writes whole 32-byte sectors.
EG2_DEV void st_global_v8(void* p, const uint32_t (&v)[8]) {
    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(v[0]), "r"(v[1]), "r"(v[2]),
                 "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}
// All but the newest N groups have finished reading their shared-memory sources.
template <int N>
EG2_DEV void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Every group of this thread has completed (writes performed).
EG2_DEV void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

EG2_DEV void tma_load_2d(void* dst, const CUtensorMap* m, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}
EG2_DEV void tma_load_3d(void* dst, const CUtensorMap* m, uint64_t* bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// ---------------------------------------------------------------------------------------------
// tcgen05
// ---------------------------------------------------------------------------------------------
// Allocate `ncols` TMEM columns (power of two >= 32); the whole warp executes this.
EG2_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(ncols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
EG2_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
EG2_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
EG2_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem], kind::f16 (bf16 inputs here), fp32 accumulation.
EG2_DEV void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// D[tmem] (+)= A[tmem] * B[smem], kind::f16: A read from tensor memory (row i in lane i, column c
// holding the K-adjacent bf16 pair (2c, 2c + 1)), B from a shared-memory descriptor.
EG2_DEV void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// Same with TF32 inputs (f32 data in shared memory).
EG2_DEV void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
template <typename TIn>
EG2_DEV void mma_bf16_or_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate);
template <>
EG2_DEV void mma_bf16_or_tf32<bf16_t>(uint32_t d, uint64_t a, uint64_t b, uint32_t i, uint32_t acc) {
    mma_bf16(d, a, b, i, acc);
}
template <>
EG2_DEV void mma_bf16_or_tf32<float>(uint32_t d, uint64_t a, uint64_t b, uint32_t i, uint32_t acc) {
    mma_tf32(d, a, b, i, acc);
}
// ---- CTA pairs (cta_group::2): one MMA over both CTAs of a 2-CTA cluster ----------------------
// M = 256: A rows 0..127 come from the issuing (even) CTA's shared memory / TMEM, rows 128..255 from
// its peer's at the same address; B is split along N (first half in the even CTA, second half in the
// odd one); D rows 0..127 land in the even CTA's TMEM, 128..255 in the odd CTA's, same columns.
// TMEM is allocated by the same warp of both CTAs.
EG2_DEV void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(ncols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::);
}
EG2_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
EG2_DEV void mma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// Copy a 128-row x 32-byte matrix (described like an MMA operand: here a 16-element K step of a
// 128-byte-swizzled K-major tile) from shared memory into TMEM lanes 0..127, 8 columns from taddr, in
// both CTAs of the pair (each from its own shared memory). Ordered with the issuing thread's MMAs.
EG2_DEV void tmem_cp_pair_128x256b(uint32_t taddr, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::2.128x256b [%0], %1;" ::"r"(taddr), "l"(sdesc));
}
EG2_DEV void mma_bf16_pair_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// Arrive on the mbarrier at shared::cluster address `bar` (either CTA of the pair) once every pair
// MMA issued so far by this thread has completed.
EG2_DEV void mma_commit_pair(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
EG2_DEV void tma_load_2d_pair(void* dst, const CUtensorMap* m, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}
// Same, arriving on the mbarrier at this shared-memory offset in both CTAs of the pair: cluster ranks
// pair_base and pair_base + 1 (pair_base = 0 in 2-CTA clusters; 0 or 2 in clusters of two pairs).
EG2_DEV void mma_commit_pair_both(uint64_t* bar, uint32_t pair_base = 0) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                     smem_u32(bar)),
                 "h"((uint16_t)(3u << pair_base))
                 : "memory");
}
// TMA tile load into this CTA's shared memory whose completion (bytes) is signalled on the mbarrier
// at shared::cluster address `bar`, which may belong to the peer CTA of the pair.
EG2_DEV void tma_load_3d_pair(void* dst, const CUtensorMap* m, uint32_t bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// Arrive on `bar` once every MMA issued so far by this thread has completed.
EG2_DEV void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane (base lane + i).
EG2_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
EG2_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]));
}
// 32 lanes x 16 consecutive 32-bit columns.
EG2_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
EG2_DEV void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]));
}
EG2_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
EG2_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

template <int W>
EG2_DEV void tmem_ldw(uint32_t taddr, uint32_t (&r)[W]) {
    if constexpr (W == 16)
        tmem_ld16(taddr, r);
    else
        tmem_ld32(taddr, r);
}
// After tcgen05.wait::ld: the registers of the waited-for loads count as written here, so no use of
// them is scheduled before the wait.
template <int W>
EG2_DEV void reg_fence(uint32_t (&r)[W]) {
#pragma unroll
    for (int j = 0; j < W; j++) asm volatile("" : "+r"(r[j]));
}
// Walks n chunks of W TMEM columns (chunk c at taddr + c * W) with the load of chunk c + 1 in flight
// while body(c, regs) processes chunk c (for loops with nothing else to hide the TMEM latency
// behind). body returns false to stop (its loads are waited for first).
template <int W, typename F>
EG2_DEV bool tmem_pipelined(uint32_t taddr, int n, F&& body) {
    uint32_t ra[W], rb[W];
    tmem_ldw<W>(taddr, ra);
#pragma unroll 1
    for (int c = 0; c < n; c += 2) {
        tmem_ld_wait();
        reg_fence<W>(ra);
        if (c + 1 < n) tmem_ldw<W>(taddr + (c + 1) * W, rb);
        if (!body(c, ra)) {
            tmem_ld_wait();
            return false;
        }
        if (c + 1 >= n) break;
        tmem_ld_wait();
        reg_fence<W>(rb);
        if (c + 2 < n) tmem_ldw<W>(taddr + (c + 2) * W, ra);
        if (!body(c + 1, rb)) {
            tmem_ld_wait();
            return false;
        }
    }
    return true;
}

// ---------------------------------------------------------------------------------------------
// UMMA descriptors
// ---------------------------------------------------------------------------------------------
// Shared-memory matrix descriptor for a tile stored with the 128-byte swizzle (rows of 128 B,
// 8-row / 1024-byte swizzle atoms, tile base 1024-byte aligned).
//   K-major operand: lbo unused (1), sbo = 1024 B between 8-row groups.
//   MN-major operand: lbo = byte stride between 64-element (128 B) chunks along M/N,
//                     sbo = 1024 B between 8-row groups along K.
EG2_DEV uint64_t umma_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version for sm_100
    d |= (uint64_t)2 << 61;  // 128-byte swizzle
    return d;
}

// Instruction descriptor: D f32, A/B format (1 = bf16, 2 = tf32), both K-major unless b_mn.
__host__ __device__ constexpr uint32_t umma_idesc(int M, int N, uint32_t ab_format, bool b_mn_major = false) {
    return (1u << 4) | (ab_format << 7) | (ab_format << 10) | ((b_mn_major ? 1u : 0u) << 16) |
           ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

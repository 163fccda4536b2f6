// Device helpers for the sm_100a kernels: mbarriers with bounded waits, 1-D
// bulk copies (TMA engine, no multicast), the m16n8k16 bf16 MMA, LOP3 and
// field reads of little-endian radix streams.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace dm {

// Device error codes written to the tensor's error word.
constexpr int kErrWaitFull = 1;    // a consumer gave up waiting for a staged unit
constexpr int kErrWaitEmpty = 2;   // the producer gave up waiting for a slot
constexpr int kErrWaitDrain = 3;   // the producer gave up draining its copies at exit
constexpr int kErrWaitPeer = 4;    // a wait for another GPU's output flag gave up

// Upper bound on polls of one mbarrier phase. Each poll suspends the warp in
// hardware for up to kSuspendNs (it resumes as soon as the phase completes),
// so a healthy wait costs one or two polls; 2^16 polls bound a wait at about
// two seconds, after which the kernel records an error and returns instead of
// waiting forever.
constexpr uint32_t kWaitPolls = 1u << 16;
// A wait for another GPU's flag: 2^23 system-scope acquire loads back to
// back (no sleep between them: that cost 0.6 % of the two-GPU step), a few
// seconds at most, then error kErrWaitPeer.
constexpr uint32_t kPeerPolls = 1u << 23;
constexpr uint32_t kSuspendNs = 32768;

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, "
        "p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "n"(kSuspendNs)
        : "memory");
    return ok != 0;
}

// Waits for the phase of `bar` with parity `parity` to complete; false
// (after writing `code` to *err) when the bound runs out.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err, int code) {
    for (uint32_t i = 0; i < kWaitPolls; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    if (err) atomicExch(err, code);
    return false;
}

// 1-D bulk copy global -> shared, completing `bytes` on `bar` (no multicast).
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Acquire / release accesses of flag words another GPU writes or reads.
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Atomic add with acquire-release semantics: the warp's earlier stores (made
// to happen before by __syncwarp) are visible to whoever acquires the new
// value, and this thread sees what the earlier releasers stored.
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t *p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void st_relaxed_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void st_relaxed_gpu(uint32_t *p, uint32_t v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Asks `bytes` (a multiple of 16, from a 16-byte aligned address) into L2.
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Retires an mbarrier so that its shared memory can be initialised again or
// reused for data (no thread waits on it and no copy completes on it).
__device__ __forceinline__ void mbar_inval(uint64_t *bar) {
    asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Orders generic-proxy accesses of global memory (e.g. another GPU's stores
// made visible by an acquire) before this thread's later bulk copies.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Orders this thread's earlier generic-proxy accesses of shared memory
// before its later async-proxy ones (a bulk copy into a slot just read).
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Programmatic dependent launch: let the next kernel in the stream start its
// CTAs (on SMs this grid leaves free) before this grid ends ...
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// ... and wait until the grid this one depends on has completed and its
// writes are visible (returns at once when there is none).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <int LUT>
__device__ __forceinline__ uint32_t lop3(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, %4;" : "=r"(d) : "r"(a), "r"(b), "r"(c), "n"(LUT));
    return d;
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + C, fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float &d0, float &d1, float &d2, float &d3, uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d0), "+f"(d1), "+f"(d2), "+f"(d3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Field `index` of a `width`-bit little-endian stream of 32-bit words.
__device__ __forceinline__ uint32_t field(const uint32_t *s, uint32_t index, uint32_t width) {
    uint32_t bit = index * width, wi = bit >> 5, lo = bit & 31;
    uint32_t v = s[wi] >> lo;
    if (lo + width > 32) v |= s[wi + 1] << (32 - lo);
    return v & ((1u << width) - 1u);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) { return __uint_as_float(b << 16); }

// Round-to-nearest-even fp32 -> bf16 bits (CUDA's conversion).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }

}  // namespace dm

// TMA (cp.async.bulk.tensor), mbarrier and work-queue helpers for the persistent
// sm_100a kernels. Every wait is bounded: on expiry the kernel records an error code in
// global memory and the caller's wait returns false instead of spinning forever.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace mwc {

// Error codes written to the workspace error word.
constexpr int ERR_WAIT_TMA = 1;     // a TMA tile never arrived
constexpr int ERR_WAIT_CHAIN = 2;   // the previous segment of a chain never published its state
constexpr int ERR_SMEM_ALIGN = 3;   // dynamic shared memory not 128-byte aligned (kernel exits)
constexpr unsigned WAIT_SPINS = 1u << 22;   // per wait: a fraction of a second with the backoff
constexpr unsigned WAIT_POLL = 1024;        // a waiting thread reads the error word this often

// True once any wait of the launch has given up: the protocol is broken, so every other
// wait returns at once instead of running to its own limit (the kernel then drains its
// loops quickly and exits normally, releasing what it holds).
__device__ __forceinline__ bool wait_aborted(const int* err) {
    return err != nullptr && *reinterpret_cast<const volatile int*>(err) != 0;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned phase) {
    unsigned ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}

// Bounded wait for an mbarrier phase; records ERR_WAIT_TMA and returns false on expiry.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned phase, int* err,
                                          unsigned limit = WAIT_SPINS) {
    for (unsigned it = 0; it < limit; ++it) {
        if (mbar_try_wait(bar, phase)) return true;
        if (it > 64) __nanosleep(32);
        if ((it & (WAIT_POLL - 1)) == WAIT_POLL - 1 && wait_aborted(err)) return false;
    }
    if (err) atomicCAS(err, 0, ERR_WAIT_TMA);
    return false;
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0,
                                             int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Orders this thread's earlier generic-proxy view of global memory (e.g. data another CTA
// published through a release / acquire flag) before its later async-proxy (bulk copy) reads.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Release / acquire flags used to hand a chain's state from one segment to the next.
__device__ __forceinline__ void flag_release(int* f, int v) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}
__device__ __forceinline__ int flag_acquire(const int* f) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
    return v;
}

// Bounded wait until *f == v; records ERR_WAIT_CHAIN and returns false on expiry.
__device__ __forceinline__ bool flag_wait(const int* f, int v, int* err) {
    for (unsigned it = 0; it < WAIT_SPINS; ++it) {
        if (flag_acquire(f) == v) return true;
        __nanosleep(it < 64 ? 20 : 200);
        if ((it & (WAIT_POLL - 1)) == WAIT_POLL - 1 && wait_aborted(err)) return false;
    }
    if (err) atomicCAS(err, 0, ERR_WAIT_CHAIN);
    return false;
}


// ---- Tensor memory (TMEM): 128 lanes x 512 columns x 32 bit per SM. A warp reaches only the
// lane quarter (warp index % 4) * 32 .. +31; an address is (lane << 16) | column. ----

// Allocate ncols columns (power of two, 32..512); one full warp issues it; the base address
// is written to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Wait for this thread's outstanding TMEM loads. The registers of a load are passed through
// so that no use of them can be scheduled before the wait.
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&v)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]),
                   "+r"(v[7]), "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]),
                   "+r"(v[14]), "+r"(v[15])
                 :);
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;"); }

// One wait for four outstanding x16 loads (all 64 registers pass through it).
__device__ __forceinline__ void tmem_wait_ld4(uint32_t (&v)[4][16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(v[0][0]), "+r"(v[0][1]), "+r"(v[0][2]), "+r"(v[0][3]), "+r"(v[0][4]), "+r"(v[0][5]),
                   "+r"(v[0][6]), "+r"(v[0][7]), "+r"(v[0][8]), "+r"(v[0][9]), "+r"(v[0][10]), "+r"(v[0][11]),
                   "+r"(v[0][12]), "+r"(v[0][13]), "+r"(v[0][14]), "+r"(v[0][15]),
                   "+r"(v[1][0]), "+r"(v[1][1]), "+r"(v[1][2]), "+r"(v[1][3]), "+r"(v[1][4]), "+r"(v[1][5]),
                   "+r"(v[1][6]), "+r"(v[1][7]), "+r"(v[1][8]), "+r"(v[1][9]), "+r"(v[1][10]), "+r"(v[1][11]),
                   "+r"(v[1][12]), "+r"(v[1][13]), "+r"(v[1][14]), "+r"(v[1][15]),
                   "+r"(v[2][0]), "+r"(v[2][1]), "+r"(v[2][2]), "+r"(v[2][3]), "+r"(v[2][4]), "+r"(v[2][5]),
                   "+r"(v[2][6]), "+r"(v[2][7]), "+r"(v[2][8]), "+r"(v[2][9]), "+r"(v[2][10]), "+r"(v[2][11]),
                   "+r"(v[2][12]), "+r"(v[2][13]), "+r"(v[2][14]), "+r"(v[2][15]),
                   "+r"(v[3][0]), "+r"(v[3][1]), "+r"(v[3][2]), "+r"(v[3][3]), "+r"(v[3][4]), "+r"(v[3][5]),
                   "+r"(v[3][6]), "+r"(v[3][7]), "+r"(v[3][8]), "+r"(v[3][9]), "+r"(v[3][10]), "+r"(v[3][11]),
                   "+r"(v[3][12]), "+r"(v[3][13]), "+r"(v[3][14]), "+r"(v[3][15]));
}

// Thread i of the warp writes / reads 16 consecutive 32-bit columns of lane (taddr lane + i).
// These touch tensor memory and registers only: no "memory" clobber, so shared / global
// loads may be scheduled across them. Their order among themselves is that of the volatile
// asm statements; tcgen05.wait::st / ::ld complete them.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
        "%12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
        "%13, %14, %15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}

}  // namespace mwc

// umma.cuh -- thin inline-PTX layer over the sm_100a tensor-core (tcgen05),
// tensor-memory (TMEM), mbarrier and bulk-copy instructions used by the
// stem kernels.  Everything here is a single instruction or a bounded wait;
// the tiling lives in the kernels.
//
// Conventions
//   * Shared-memory operands use the K-major, no-swizzle canonical layout:
//     a "core matrix" is 8 rows x 16 bytes stored as 128 contiguous bytes
//     (row r at +16*r); the two core matrices of one K=16 step sit LBO bytes
//     apart; consecutive 8-row groups along M (or N) sit SBO bytes apart.
//     With SBO = 128 every row of the operand is simply 16 bytes after the
//     previous one, so an operand shifted by s rows is the same descriptor
//     with the start address moved by 16*s bytes -- which is how the 3x3x3
//     conv taps are expressed without any im2col copy.
//   * TMEM addresses are (lane << 16) | column.  Warp w of a warpgroup may
//     only touch lanes [32*(w%4), 32*(w%4)+32).
//   * Every wait is bounded (kWaitRounds suspended polls); on expiry it returns false
//     and the caller records an error and winds down instead of hanging.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace ww {
namespace umma {


__device__ __forceinline__ uint32_t smem_addr(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// Descriptors
// ---------------------------------------------------------------------------

// Shared-memory matrix descriptor, K-major, SWIZZLE_NONE, sm_100 version 1.
// Bits: [0,14) start>>4, [16,30) LBO>>4, [32,46) SBO>>4, [46,48) version=1,
// [49,52) base offset = 0, [52] LBO mode = 0, [61,64) layout = 0 (none).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo)
{
    return (static_cast<uint64_t>((saddr >> 4) & 0x3FFFu)) |
           (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) |
           (static_cast<uint64_t>(1u) << 46);
}

// Adding a byte offset to a descriptor's start address (offset % 16 == 0;
// the 14-bit field never carries for shared addresses < 256 KB).
__device__ __forceinline__ uint64_t desc_advance(uint64_t desc, uint32_t byte_offset)
{
    return desc + static_cast<uint64_t>(byte_offset >> 4);
}

// Instruction descriptor for kind::f16 with fp16 A and B, fp32 accumulate,
// both operands K-major, dense.  N % 16 == 0 for M == 128.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N)
{
    return (1u << 4)                                    // D format: f32
           | (0u << 7)                                  // A format: f16
           | (0u << 10)                                 // B format: f16
           | (static_cast<uint32_t>(N >> 3) << 17)      // N / 8
           | (static_cast<uint32_t>(M >> 4) << 24);     // M / 16
}

// ---------------------------------------------------------------------------
// MMA issue (one thread) and completion tracking
// ---------------------------------------------------------------------------

// D[tmem] (+)= A[smem] * B[smem]^T, one K=16 step.  No "memory" clobber:
// operand visibility is ordered by fences + mbarriers, and leaving ordinary
// loads free to move lets the compiler prefetch the next descriptors.
__device__ __forceinline__ void mma_f16_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
        :
        : "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Arrive (once) on an mbarrier when every MMA issued so far by this thread
// has completed.
__device__ __forceinline__ void mma_commit(uint32_t mbar_saddr)
{
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n"
        :
        : "r"(mbar_saddr)
        : "memory");
}

__device__ __forceinline__ void fence_before_sync()
{
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}

__device__ __forceinline__ void fence_after_sync()
{
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}

// Make this thread's generic-proxy shared-memory writes visible to the
// async proxy (tensor-core operand reads, bulk copies).
__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMEM allocation (whole warp)
// ---------------------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t dst_saddr, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n"
                 :
                 : "r"(dst_saddr), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n"
                 :
                 : "r"(taddr), "r"(ncols)
                 : "memory");
}

// ---------------------------------------------------------------------------
// TMEM -> registers (whole warp; each thread gets its own lane)
// ---------------------------------------------------------------------------

// 16 consecutive 32-bit columns of this thread's lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
          "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
          "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// 8 consecutive 32-bit columns of this thread's lane.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
          "=r"(r[6]), "=r"(r[7])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld()
{
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

// 8 consecutive 32-bit columns of this thread's lane <- registers.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n"
        :
        : "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
          "r"(r[6]), "r"(r[7])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_st()
{
    asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint32_t saddr, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" : : "r"(saddr), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t saddr)
{
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}\n"
                 :
                 : "r"(saddr)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t saddr, uint32_t bytes)
{
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}\n"
                 :
                 : "r"(saddr), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t saddr, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(saddr), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking poll: has the phase with the given parity completed?
// (try_wait may suspend the thread for a system-defined time when it has
// not; a polling loop that interleaves other work must use test_wait.)
__device__ __forceinline__ bool mbar_test_wait(uint32_t saddr, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(saddr), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait that lets the hardware suspend the thread for up to `hint_ns`
// nanoseconds (it resumes as soon as the phase completes), so waiting warps
// do not spin through issue slots the working warps need.
__device__ __forceinline__ bool mbar_try_wait_hint(uint32_t saddr, uint32_t parity, uint32_t hint_ns)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(saddr), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity to complete: at most
// kWaitRounds suspended polls of <= 1 ms each (seconds in total, orders of
// magnitude above any legitimate wait in these kernels).
constexpr uint32_t kWaitRounds = 4000;
constexpr uint32_t kSpinPolls = 4;   // non-blocking polls before suspending (64 polling warps slowed config 3 by 8 %)
__device__ __forceinline__ bool mbar_wait(uint32_t saddr, uint32_t parity)
{
    for (uint32_t i = 0; i < kSpinPolls; ++i)
        if (mbar_test_wait(saddr, parity)) return true;
    for (uint32_t i = 0; i < kWaitRounds; ++i)
        if (mbar_try_wait_hint(saddr, parity, 1000000u)) return true;
    return false;
}

// ---------------------------------------------------------------------------
// Bulk copies (TMA engine, untiled) global -> shared and shared -> global
// ---------------------------------------------------------------------------

// Both addresses 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(uint32_t dst_saddr, const void* src, uint32_t bytes,
                                         uint32_t mbar_saddr)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
        :
        : "r"(dst_saddr), "l"(src), "r"(bytes), "r"(mbar_saddr)
        : "memory");
}

}  // namespace umma
}  // namespace ww

namespace ww {
namespace umma {

// 3-D tiled TMA load global -> shared, completion counted on an mbarrier.
// `tmap` is the generic address of a CUtensorMap kernel parameter.
// Coordinates are element indices (x innermost); x * sizeof(elem) must be a
// multiple of 16 bytes; out-of-range elements are filled with zeros.
__device__ __forceinline__ void tma_load_3d(uint32_t dst_saddr, const void* tmap, int x, int y, int z,
                                            uint32_t mbar_saddr)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4}], [%5];\n"
        :
        : "r"(dst_saddr), "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(mbar_saddr)
        : "memory");
}

// 4-D tiled TMA load global -> shared (this CTA), completion counted on an
// mbarrier; same coordinate rules as tma_load_3d.
__device__ __forceinline__ void tma_load_4d(uint32_t dst_saddr, const void* tmap, int x, int y, int z, int w,
                                            uint32_t mbar_saddr)
{
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4, %5}], [%6];\n"
        :
        : "r"(dst_saddr), "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(w), "r"(mbar_saddr)
        : "memory");
}

// 5-D tiled TMA load global -> shared (this CTA); same rules as tma_load_3d.
__device__ __forceinline__ void tma_load_5d(uint32_t dst_saddr, const void* tmap, int x, int y, int z, int w, int v,
                                            uint32_t mbar_saddr)
{
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4, %5, %6}], [%7];\n"
        :
        : "r"(dst_saddr), "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(w), "r"(v), "r"(mbar_saddr)
        : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const void* tmap)
{
    asm volatile("prefetch.tensormap [%0];\n" : : "l"(tmap) : "memory");
}

// fp32 result of fp16 * fp16 + fp32 with a single rounding: identical to
// fmaf((float)a, (float)b, c) because the product of two fp16 values is
// exact in fp32.
__device__ __forceinline__ float fma_f16f16f32(unsigned short a, unsigned short b, float c)
{
    float d;
    asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
    return d;
}

// ---- warp-level (mma.sync) helpers for small banded tiles ----

__device__ __forceinline__ unsigned short ld_shared_u16(uint32_t saddr)
{
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];\n" : "=h"(v) : "r"(saddr));
    return v;
}

__device__ __forceinline__ uint32_t pack_b16x2(unsigned short lo, unsigned short hi)
{
    uint32_t r;
    asm("mov.b32 %0, {%1, %2};\n" : "=r"(r) : "h"(lo), "h"(hi));
    return r;
}

__device__ __forceinline__ void unpack_b16x2(uint32_t v, unsigned short& lo, unsigned short& hi)
{
    asm("mov.b32 {%0, %1}, %2;\n" : "=h"(lo), "=h"(hi) : "r"(v));
}

__device__ __forceinline__ void st_shared_u16(uint32_t saddr, unsigned short v)
{
    asm volatile("st.shared.u16 [%0], %1;\n" : : "r"(saddr), "h"(v) : "memory");
}

__device__ __forceinline__ void ld_shared_v4(uint32_t saddr, uint32_t (&v)[4])
{
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];\n"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(saddr)
                 : "memory");
}

__device__ __forceinline__ void st_shared_v4(uint32_t saddr, uint32_t a, uint32_t b, uint32_t c, uint32_t d)
{
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};\n" : : "r"(saddr), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}

// Four 8x8 b16 matrices, transposed: lanes 8i..8i+7 give the row addresses
// of matrix i; register i receives its fragment (thread t: rows 2(t%4) and
// 2(t%4)+1 of column t/4).
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t saddr, uint32_t (&r)[4])
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(saddr));
}

// D = A (16x8, row) * B (8x8, col) + D, fp16 inputs, fp32 accumulators.
__device__ __forceinline__ void mma_16x8x8_f16f32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0)
{
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5}, {%6}, "
                 "{%0, %1, %2, %3};\n"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(b0));
}

// D = A (16x16, row) * B (16x8, col) + D, fp16 inputs, fp32 accumulators.
__device__ __forceinline__ void mma_16x8x16_f16f32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                   uint32_t a3, uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
                 "{%8, %9}, {%0, %1, %2, %3};\n"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

}  // namespace umma
}  // namespace ww

// corr_volume.cu -- group-wise stereo correlation volume (CorrVolume).
//
//   out[b, g, d, h, w] = scale( sum_{c in group g} L[b,c,h,w] * R[b,c,h,w-d] ),  +0 if w-d < 0
//
// Semantics follow the reference kernels exactly (corr_volume_kernel.cu:52-88
// naive, :118-239 fast): an fp32 fma chain over the group's channels in
// channel order starting from +0, then either acc / C (what the naive kernel
// does) or acc * (1/C) (what the fast kernel does), rounded to the output
// type.  Which of the two the reference would have used for the equivalent
// call is decided on the host (corr_scale_mode) so results are bit-identical
// to the reference called once per (b, g).
//
// B200 design.  The op is HBM-bound: it reads L and R once and writes G*D
// output values per input pixel per group.  One CTA owns one image row
// segment of 128 columns (64 or 32 when the image is that narrow) for one
// (b, g) and a band of DT disparities (fewer when the grid would not fill
// the SMs twice):
//   * the group's L row segment [w0, w0+128) and the matching R segment
//     [w0 - d0 - DT, w0 - d0 + 128) are staged channel-chunk by chunk into
//     shared memory with 16-byte vector loads (zero fill off the image, which
//     is also the w-d<0 padding);
//   * each thread keeps a 4-column x 8-disparity register tile: per channel
//     4 L loads + 11 R loads feed 32 fma, so the shared pipe is not the limit;
//   * each warp writes 4 contiguous columns per thread -> 256 B coalesced
//     stores per disparity row.
// Grid: x = column tiles (fastest, so neighbouring tiles share R in L2),
// y = row x disparity band, z = batch x group.
// Volumes too small to fill the SMs with such tiles (the reference's native
// 1 x 48 x 32 x 40 among them) run corr_volume_small_kernel instead: one
// thread per output, operands through L2.

#include "int_div.cuh"
#include "ww_common.cuh"

#include <type_traits>

namespace ww {
namespace {

constexpr int kTileW = 128;     // widest column tile per CTA (32 threads x 4); 64 and 32 for narrow images
constexpr int kVecW = 4;        // columns per thread
constexpr int kDispPerThread = 8;
constexpr int kChunkC = 16;     // channels staged per pass (32 with the narrow tiles)
constexpr int kSmallOutputsPerSM = 800;  // below this many outputs per SM: one thread per output
constexpr int kRuleDivide = 1;           // row-streaming kernels: scale by rounded division
constexpr int kRuleZero = 2;             //   and an explicit +0 where w - d < 0 (the naive rule)

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }

// Stage rows [c0, c0+nc) x columns [col0, col0+width) of one (b, h) image row
// into smem[nc][width], zero outside [0, W).  Each thread issues its loads in
// batches of NB 16-byte vectors before storing any of them, so a chunk costs
// one memory latency per batch rather than one per vector (the narrow tiles,
// whose few threads stage ~13 vectors per chunk).
template <typename T, int NB>
__device__ __forceinline__ void stage_rows_batched(T* __restrict__ dst, const T* __restrict__ src_row0,
                                           int64_t chan_stride, int nc, int col0, int width, int W,
                                           bool vec_ok)
{
    constexpr int kVec = 16 / sizeof(T);
    const int nvec = width / kVec;  // width is a multiple of kVec
    const int nthr = blockDim.x * blockDim.y;
    const int t = threadIdx.y * blockDim.x + threadIdx.x;
    for (int base = 0; base < nc * nvec; base += NB * nthr) {
        uint4 v[NB];
#pragma unroll
        for (int k = 0; k < NB; ++k) {
            const int i = base + k * nthr + t;
            v[k] = make_uint4(0u, 0u, 0u, 0u);  // zero in both fp16 and fp32
            if (i < nc * nvec) {
                const int c = i / nvec;
                const int gx = col0 + (i - c * nvec) * kVec;
                const T* src = src_row0 + c * chan_stride;
                if (vec_ok && gx >= 0 && gx + kVec <= W) {
                    v[k] = __ldg(reinterpret_cast<const uint4*>(src + gx));
                } else {
                    T e[kVec];
#pragma unroll
                    for (int q = 0; q < kVec; ++q) {
                        const int g = gx + q;
                        e[q] = (g >= 0 && g < W) ? src[g] : from_f32<T>(0.0f);
                    }
                    v[k] = *reinterpret_cast<const uint4*>(e);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < NB; ++k) {
            const int i = base + k * nthr + t;
            if (i < nc * nvec) *reinterpret_cast<uint4*>(dst + i * kVec) = v[k];
        }
    }
}

// The same with one vector per loop trip (the 128-column tiles: measured
// faster there than the batched form, whose registers cost occupancy).
template <typename T>
__device__ __forceinline__ void stage_rows_loop(T* __restrict__ dst, const T* __restrict__ src_row0,
                                                int64_t chan_stride, int nc, int col0, int width, int W,
                                                bool vec_ok)
{
    constexpr int kVec = 16 / sizeof(T);
    const int nvec = width / kVec;  // width is a multiple of kVec
    for (int i = threadIdx.y * blockDim.x + threadIdx.x; i < nc * nvec; i += blockDim.x * blockDim.y) {
        const int c = i / nvec;
        const int x = (i - c * nvec) * kVec;
        const int gx = col0 + x;
        const T* src = src_row0 + c * chan_stride;
        T* d = dst + c * width + x;
        if (vec_ok && gx >= 0 && gx + kVec <= W) {
            *reinterpret_cast<uint4*>(d) = __ldg(reinterpret_cast<const uint4*>(src + gx));
        } else {
#pragma unroll
            for (int k = 0; k < kVec; ++k) {
                const int g = gx + k;
                d[k] = (g >= 0 && g < W) ? src[g] : from_f32<T>(0.0f);
            }
        }
    }
}

template <typename T, int TW>
__device__ __forceinline__ void stage_rows(T* __restrict__ dst, const T* __restrict__ src_row0,
                                           int64_t chan_stride, int nc, int col0, int width, int W,
                                           bool vec_ok)
{
    if constexpr (TW == kTileW) stage_rows_loop<T>(dst, src_row0, chan_stride, nc, col0, width, W, vec_ok);
    else stage_rows_batched<T, 8>(dst, src_row0, chan_stride, nc, col0, width, W, vec_ok);
}

__device__ __forceinline__ void unpack_h2(uint32_t x, unsigned short& lo, unsigned short& hi)
{
    asm("mov.b32 {%0, %1}, %2;" : "=h"(lo), "=h"(hi) : "r"(x));
}

// fp32 a * b + c of two fp16 operands with one rounding (the product is
// exact in fp32): the same value as fmaf(float(a), float(b), c).
__device__ __forceinline__ float fma_h(unsigned short a, unsigned short b, float c)
{
    float d;
    asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
    return d;
}

template <typename T, int TW, int CC>
__global__ void __launch_bounds__(256) corr_volume_kernel(
    const T* __restrict__ left, const T* __restrict__ right, T* __restrict__ out,
    int C, int H, int W, int D, int G, int n_dband, int scale_div, float inv_cg, int vec_ok)
{
    constexpr int ND = TW == kTileW ? kDispPerThread : kDispPerThread / 2;
    const int DT = ND * blockDim.y;  // disparities per CTA
    const int RW = TW + DT;      // staged R width
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* Ls = reinterpret_cast<T*>(smem_raw);
    T* Rs = Ls + CC * TW;

    const int w0 = blockIdx.x * TW;
    const int h = blockIdx.y / n_dband;
    const int d0 = (blockIdx.y - h * n_dband) * DT;
    const int b = blockIdx.z / G;
    const int g = blockIdx.z - b * G;
    const int Cg = C / G;

    const int64_t plane = i64(H) * W;
    const T* lrow = left + (i64(b) * C + i64(g) * Cg) * plane + i64(h) * W;
    const T* rrow = right + (i64(b) * C + i64(g) * Cg) * plane + i64(h) * W;

    const int wl = threadIdx.x * kVecW;
    const int dd0 = threadIdx.y * ND;
    // R index of (v = 0, dd = ND-1): rl = wl + v - (dd0 + dd) + DT.
    const int rbase = wl - dd0 + DT - (ND - 1);

    float acc[ND][kVecW];
#pragma unroll
    for (int i = 0; i < ND; ++i)
#pragma unroll
        for (int v = 0; v < kVecW; ++v) acc[i][v] = 0.0f;

    for (int c0 = 0; c0 < Cg; c0 += CC) {
        const int nc = min(CC, Cg - c0);
        stage_rows<T, TW>(Ls, lrow + c0 * plane, plane, nc, w0, TW, W, vec_ok);
        stage_rows<T, TW>(Rs, rrow + c0 * plane, plane, nc, w0 - d0 - DT, RW, W, vec_ok);
        __syncthreads();
        for (int c = 0; c < nc; ++c) {
            const T* lp = Ls + c * TW + wl;
            const T* rp = Rs + c * RW + rbase;
            float lv[kVecW], rv[ND + kVecW - 1];
#pragma unroll
            for (int v = 0; v < kVecW; ++v) lv[v] = to_f32<T>(lp[v]);
#pragma unroll
            for (int k = 0; k < ND + kVecW - 1; ++k) rv[k] = to_f32<T>(rp[k]);
#pragma unroll
            for (int dd = 0; dd < ND; ++dd)
#pragma unroll
                for (int v = 0; v < kVecW; ++v)
                    acc[dd][v] = __fmaf_rn(lv[v], rv[(ND - 1) - dd + v], acc[dd][v]);
        }
        __syncthreads();
    }

    T* obase = out + (i64(b) * G + g) * i64(D) * plane + i64(h) * W;
    const int gx = w0 + wl;
#pragma unroll
    for (int dd = 0; dd < ND; ++dd) {
        const int d = d0 + dd0 + dd;
        if (d >= D) break;
        T* op = obase + i64(d) * plane + gx;
        T tmp[kVecW];
#pragma unroll
        for (int v = 0; v < kVecW; ++v) {
            float val;
            if (gx + v < d) val = 0.0f;  // w - d < 0: exact +0
            else val = scale_div ? div_int(acc[dd][v], Cg, inv_cg) : __fmul_rn(acc[dd][v], inv_cg);
            tmp[v] = from_f32<T>(val);
        }
        if (gx + kVecW <= W && (reinterpret_cast<uintptr_t>(op) % (kVecW * sizeof(T))) == 0) {
            if constexpr (sizeof(T) == 2) *reinterpret_cast<uint2*>(op) = *reinterpret_cast<uint2*>(tmp);
            else *reinterpret_cast<uint4*>(op) = *reinterpret_cast<uint4*>(tmp);
        } else {
#pragma unroll
            for (int v = 0; v < kVecW; ++v)
                if (gx + v < W) op[v] = tmp[v];
        }
    }
}

// fp16 images wider than 64 columns.  Same register tile (4 columns x 8
// disparities per thread, fp32 fma chains in channel order from +0) as
// corr_volume_kernel, with three changes that cut the instructions per fma
// from about two to about one:
//   * the column tile is sized to the image (tw = W / ceil(W / 256) rounded
//     up to 16: one 160-column tile for W = 160, two for W = 312), not fixed
//     at 128 columns, which left most of a second tile idle;
//   * per channel the 4 left and 11 right operands come in as one and three
//     8-byte shared loads (the right ones from the 4-aligned position one
//     before the first needed);
//   * the fma takes the fp16 operands directly (fma.rn.f32.f16: the product
//     of two fp16 values is exact in fp32, so the result is identical to
//     converting them first), so no conversions are issued.
// blockDim = (tw / 4, ny), ny * 8 = DT disparities per CTA.
template <int CC>
__global__ void __launch_bounds__(512) corr_volume_h_kernel(
    const __half* __restrict__ left, const __half* __restrict__ right, __half* __restrict__ out,
    int C, int H, int W, int D, int G, int n_dband, int tw, int scale_div, float inv_cg, int vec_ok)
{
    constexpr int ND = kDispPerThread;
    const int DT = ND * blockDim.y;
    const int RW = tw + DT;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __half* Ls = reinterpret_cast<__half*>(smem_raw);
    __half* Rs = Ls + CC * tw;

    const int w0 = blockIdx.x * tw;
    const int h = blockIdx.y / n_dband;
    const int d0 = (blockIdx.y - h * n_dband) * DT;
    const int b = blockIdx.z / G;
    const int g = blockIdx.z - b * G;
    const int Cg = C / G;

    const int64_t plane = i64(H) * W;
    const __half* lrow = left + (i64(b) * C + i64(g) * Cg) * plane + i64(h) * W;
    const __half* rrow = right + (i64(b) * C + i64(g) * Cg) * plane + i64(h) * W;

    const int wl = threadIdx.x * kVecW;
    const int dd0 = threadIdx.y * ND;
    // First of the 12 staged right values loaded per channel: the value
    // for (column wl, disparity dd0 + ND - 1) is one after it.
    const int rs = wl - dd0 + DT - ND;

    float acc[ND][kVecW];
#pragma unroll
    for (int i = 0; i < ND; ++i)
#pragma unroll
        for (int v = 0; v < kVecW; ++v) acc[i][v] = 0.0f;

    for (int c0 = 0; c0 < Cg; c0 += CC) {
        const int nc = min(CC, Cg - c0);
        stage_rows_loop<__half>(Ls, lrow + c0 * plane, plane, nc, w0, tw, W, vec_ok);
        stage_rows_loop<__half>(Rs, rrow + c0 * plane, plane, nc, w0 - d0 - DT, RW, W, vec_ok);
        __syncthreads();
        for (int c = 0; c < nc; ++c) {
            const uint2 l4 = *reinterpret_cast<const uint2*>(Ls + c * tw + wl);
            const __half* rp = Rs + c * RW + rs;
            const uint2 r0 = *reinterpret_cast<const uint2*>(rp);
            const uint2 r1 = *reinterpret_cast<const uint2*>(rp + 4);
            const uint2 r2 = *reinterpret_cast<const uint2*>(rp + 8);
            unsigned short lv[kVecW], rv[12];
            unpack_h2(l4.x, lv[0], lv[1]);
            unpack_h2(l4.y, lv[2], lv[3]);
            unpack_h2(r0.x, rv[0], rv[1]);
            unpack_h2(r0.y, rv[2], rv[3]);
            unpack_h2(r1.x, rv[4], rv[5]);
            unpack_h2(r1.y, rv[6], rv[7]);
            unpack_h2(r2.x, rv[8], rv[9]);
            unpack_h2(r2.y, rv[10], rv[11]);
#pragma unroll
            for (int dd = 0; dd < ND; ++dd)
#pragma unroll
                for (int v = 0; v < kVecW; ++v)
                    acc[dd][v] = fma_h(lv[v], rv[ND - dd + v], acc[dd][v]);
        }
        __syncthreads();
    }

    __half* obase = out + (i64(b) * G + g) * i64(D) * plane + i64(h) * W;
    const int gx = w0 + wl;
    if (gx >= W) return;
#pragma unroll
    for (int dd = 0; dd < ND; ++dd) {
        const int d = d0 + dd0 + dd;
        if (d >= D) break;
        __half* op = obase + i64(d) * plane + gx;
        __half tmp[kVecW];
#pragma unroll
        for (int v = 0; v < kVecW; ++v) {
            float val;
            if (gx + v < d) val = 0.0f;  // w - d < 0: exact +0
            else val = scale_div ? div_int(acc[dd][v], Cg, inv_cg) : __fmul_rn(acc[dd][v], inv_cg);
            tmp[v] = __float2half_rn(val);
        }
        if (gx + kVecW <= W && (reinterpret_cast<uintptr_t>(op) % 8) == 0) {
            *reinterpret_cast<uint2*>(op) = *reinterpret_cast<uint2*>(tmp);
        } else {
#pragma unroll
            for (int v = 0; v < kVecW; ++v)
                if (gx + v < W) op[v] = tmp[v];
        }
    }
}

// cp.async staging of rows [0, nc) x columns [col0, col0 + width) of one
// image row into dst[nc][width] (16-byte vectors; W % 8 == 0 and 16-byte
// aligned bases, so a vector is wholly inside or wholly outside the image;
// outside ones are zero-filled by the copy itself).  Not waited for here.
__device__ __forceinline__ void stage_rows_async(__half* dst, const __half* src_row0, int64_t chan_stride, int nc,
                                                 int col0, int width, int W)
{
    const int nvec = width / 8;
    for (int i = threadIdx.y * blockDim.x + threadIdx.x; i < nc * nvec; i += blockDim.x * blockDim.y) {
        const int c = i / nvec;
        const int x = (i - c * nvec) * 8;
        const int gx = col0 + x;
        const bool in = gx >= 0 && gx < W;
        const __half* src = src_row0 + c * chan_stride + (in ? gx : 0);
        const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst + c * width + x));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" : : "r"(d), "l"(src), "r"(in ? 16 : 0)
                     : "memory");
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
}

// (x * s, y * s) with one packed fp32 multiply (each lane rounded as
// __fmul_rn) and one packed round to fp16 (each as __float2half_rn).
__device__ __forceinline__ uint32_t scale2_to_half2(float x, float y, float s)
{
    uint64_t v, sv, r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "f"(x), "f"(y));
    asm("mov.b64 %0, {%1, %1};" : "=l"(sv) : "f"(s));
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(v), "l"(sv));
    float a, b;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
    const __half2 h2 = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h2);
}

// The general epilogue of one disparity's VW columns (gx .. gx + VW - 1) of a
// row-streaming register tile under scale rule RULE, as packed fp16 pairs:
// acc / Cg (kRuleDivide: the correction step of int_div.cuh for every value)
// or acc * (1 / Cg), and, under kRuleZero, an explicit +0 where w - d < 0
// (specialising the tiles that never reach w - d < 0 was measured slower:
// config 3 162 against 138 us).  Returns whether some value was outside
// the correction step's exact range; the caller then rewrites its tile with
// corr_rows_exact, so the common path has no per-value branch.  For fp16
// features that range test is a finiteness test: every product of two fp16
// values is exact in fp32 and a multiple of 2^-48, so is every fp32 partial
// sum of them (rounding a multiple of 2^-48 to fp32 gives one again), hence a
// sum is 0 or at least 2^-48 in magnitude (never in (0, 2^-100)), and Cg
// products of at most 65504^2 stay finite unless an input is infinite or NaN.
template <int VW, int RULE>
__device__ __forceinline__ bool scale_cols(const float (&acc)[VW], int gx, int d, int Cg, float inv_cg,
                                           uint32_t (&h)[VW / 2])
{
    bool redo = false;
#pragma unroll
    for (int v = 0; v < VW; v += 2) {
        float q[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const float a = acc[v + k];
            if constexpr ((RULE & kRuleDivide) != 0) {
                q[k] = div_by_int_core(a, static_cast<float>(Cg), inv_cg);
                redo |= !(fabsf(a) <= 0x1.fffffep127f);  // infinite or NaN (see above)
            } else {
                q[k] = __fmul_rn(a, inv_cg);
            }
            if ((RULE & kRuleZero) != 0 && gx + v + k < d) q[k] = 0.0f;  // naive rule: w - d < 0 is +0
        }
        const __half2 h2 = __floats2half2_rn(q[0], q[1]);
        h[v / 2] = *reinterpret_cast<const uint32_t*>(&h2);
    }
    return redo;
}

// The rare path of the divide rule: a thread whose tile held a value outside
// the correction step's range recomputes its ND x VW outputs from the staged
// row (the same fp32 fma chain in channel order from +0, so the same sums),
// divides with div_int and stores them one by one over what it stored.
// Not inlined: the common path keeps the registers the division subroutine
// would need.
template <int VW>
__device__ __noinline__ void corr_rows_exact(const __half* Ls, const __half* Rs, int tw, int RW, int wl, int rs,
                                             int Cg, float inv_cg, int dd0, int D, int gx, int W, bool zero_rule,
                                             __half* op, int64_t plane)
{
    constexpr int ND = kDispPerThread;
    const unsigned short* L = reinterpret_cast<const unsigned short*>(Ls);
    const unsigned short* R = reinterpret_cast<const unsigned short*>(Rs);
    for (int dd = 0; dd < ND && dd0 + dd < D; ++dd)
        for (int v = 0; v < VW && gx + v < W; ++v) {
            float a = 0.0f;
            for (int c = 0; c < Cg; ++c) a = fma_h(L[c * tw + wl + v], R[c * RW + rs + ND - dd + v], a);
            float q = div_int(a, Cg, inv_cg);
            if (zero_rule && gx + v < dd0 + dd) q = 0.0f;
            op[dd * plane + v] = __float2half_rn(q);
        }
}

// fp16, W > 64, W % 8 == 0, the group's channels in one staged chunk
// (Cg <= CC) and all disparities in one band.  The register tile and the
// arithmetic are corr_volume_h_kernel's (4 columns x 8 disparities per
// thread, fp32 fma chains in channel order from +0, the same scale rule and
// rounding), so the results are bit-identical.  Two changes:
//   * a CTA streams `rows` consecutive image rows of one (b, g, column
//     tile) through a ring of three row buffers: row h + 2's left and right
//     segments are copied in (cp.async, zero fill off the image) while row h
//     is computed and stored, so only the first row waits for its copy, one
//     barrier per row suffices, and the grid is about one wave of resident
//     CTAs;
//   * the epilogue costs about 1.5 instructions per output instead of 4 for
//     threads whose 8 disparities are all <= their first column (no w - d < 0
//     test; scale and fp16 rounding packed two values at a time): with Cg = 8
//     a value takes only 8 fmas, so the epilogue was most of the
//     instructions (measured).
// Measured alternatives that were slower: fp32 copies of the staged rows
// (one conversion per staged value instead of per use: more registers,
// fewer CTAs), bulk-copy (TMA engine) staging of the 2 Cg row segments
// from one thread, and selecting the w - d < 0 zeros before a shared
// packed epilogue.
// CG: channels per group when known at compile time (the channel loop is
// then unrolled with immediate offsets), 0 otherwise.  RULE: the scale rule
// (kRuleDivide | kRuleZero bits), a compile-time constant so the epilogue
// carries no per-value rule tests.  64 registers: 4 CTAs of 240 threads per
// SM (measured faster than 80 registers and 3 CTAs on every benchmark shape
// but config 2, where it is 4 % slower).
template <int CC, int CG, int RULE>
__global__ void __maxnreg__(64) corr_volume_rows_kernel(
    const __half* __restrict__ left, const __half* __restrict__ right, __half* __restrict__ out,
    int C, int H, int W, int D, int G, int rows, int tw, float inv_cg)
{
    constexpr int ND = kDispPerThread;
    const int DT = ND * blockDim.y;
    const int RW = tw + DT;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __half* buf = reinterpret_cast<__half*>(smem_raw);
    const int buf_elems = CC * (tw + RW);

    const int w0 = blockIdx.x * tw;
    const int h0 = blockIdx.y * rows;
    const int h1 = min(h0 + rows, H);
    const int b = blockIdx.z / G;
    const int g = blockIdx.z - b * G;
    const int Cg = CG > 0 ? CG : C / G;
    const int64_t plane = i64(H) * W;
    const __half* lbase = left + (i64(b) * C + i64(g) * Cg) * plane;
    const __half* rbase = right + (i64(b) * C + i64(g) * Cg) * plane;

    const int wl = threadIdx.x * kVecW;
    const int dd0 = threadIdx.y * ND;
    const int rs = wl - dd0 + DT - ND;
    const int gx = w0 + wl;
    // Packed epilogue when all 8 disparities exist, all 4 columns are inside
    // the image, no division is needed and no output needs the naive rule's
    // zero.  Under the fast rule the reference kernel
    // (corr_volume_kernel.cu:220-228) writes acc * (1/C) for w - d < 0 too,
    // from right columns staged as zeros: +0 for finite features, exactly
    // what the zero-filled staging gives here, so those outputs need no test.
    // Under the naive rule (:75-86) they are an explicit +0.
    // RULE: kRuleDivide (acc / Cg; otherwise * (1 / Cg), the same when Cg
    // is a power of two) | kRuleZero (the naive rule's explicit +0).
    constexpr bool divide = (RULE & kRuleDivide) != 0;
    constexpr bool zero_rule = (RULE & kRuleZero) != 0;
    const bool plain = dd0 + ND <= D && gx + kVecW <= W && !divide && !(zero_rule && gx < dd0 + ND - 1);
    __half* obase = out + ((i64(b) * G + g) * D + dd0) * plane + gx;

    auto stage = [&](int hh) {
        __half* nL = buf + ((hh - h0) % 3) * buf_elems;
        stage_rows_async(nL, lbase + i64(hh) * W, plane, Cg, w0, tw, W);
        stage_rows_async(nL + CC * tw, rbase + i64(hh) * W, plane, Cg, w0 - DT, RW, W);
    };
    if (h0 < h1) stage(h0);
    if (h0 + 1 < h1) stage(h0 + 1);
    for (int h = h0; h < h1; ++h) {
        const __half* Ls = buf + ((h - h0) % 3) * buf_elems;
        const __half* Rs = Ls + CC * tw;
        if (h + 1 < h1) asm volatile("cp.async.wait_group 2;\n" ::: "memory");
        else asm volatile("cp.async.wait_group 0;\n" ::: "memory");
        __syncthreads();  // row h landed for every thread; row h - 1's compute done everywhere
        if (h + 2 < h1) stage(h + 2);  // into row h - 1's buffer
        float acc[ND][kVecW];
#pragma unroll
        for (int i = 0; i < ND; ++i)
#pragma unroll
            for (int v = 0; v < kVecW; ++v) acc[i][v] = 0.0f;
#pragma unroll(CG > 0 ? CG : 1)
        for (int c = 0; c < Cg; ++c) {
            const uint2 l4 = *reinterpret_cast<const uint2*>(Ls + c * tw + wl);
            const __half* rp = Rs + c * RW + rs;
            const uint2 r0 = *reinterpret_cast<const uint2*>(rp);
            const uint2 r1 = *reinterpret_cast<const uint2*>(rp + 4);
            const uint2 r2 = *reinterpret_cast<const uint2*>(rp + 8);
            unsigned short lv[kVecW], rv[12];
            unpack_h2(l4.x, lv[0], lv[1]);
            unpack_h2(l4.y, lv[2], lv[3]);
            unpack_h2(r0.x, rv[0], rv[1]);
            unpack_h2(r0.y, rv[2], rv[3]);
            unpack_h2(r1.x, rv[4], rv[5]);
            unpack_h2(r1.y, rv[6], rv[7]);
            unpack_h2(r2.x, rv[8], rv[9]);
            unpack_h2(r2.y, rv[10], rv[11]);
#pragma unroll
            for (int dd = 0; dd < ND; ++dd)
#pragma unroll
                for (int v = 0; v < kVecW; ++v) acc[dd][v] = fma_h(lv[v], rv[ND - dd + v], acc[dd][v]);
        }
        __half* op = obase + i64(h) * W;
        if (plain) {
#pragma unroll
            for (int dd = 0; dd < ND; ++dd) {
                uint2 u;
                u.x = scale2_to_half2(acc[dd][0], acc[dd][1], inv_cg);
                u.y = scale2_to_half2(acc[dd][2], acc[dd][3], inv_cg);
                *reinterpret_cast<uint2*>(op + dd * plane) = u;
            }
        } else if (gx < W) {
            bool redo = false;
#pragma unroll
            for (int dd = 0; dd < ND; ++dd) {
                const int d = dd0 + dd;
                if (d >= D) break;
                uint32_t hv[kVecW / 2];
                redo |= scale_cols<kVecW, RULE>(acc[dd], gx, d, Cg, inv_cg, hv);
                __half* o = op + dd * plane;
                if (gx + kVecW <= W) {
                    *reinterpret_cast<uint2*>(o) = make_uint2(hv[0], hv[1]);
                } else {
#pragma unroll
                    for (int v = 0; v < kVecW; ++v)
                        if (gx + v < W)
                            o[v] = __ushort_as_half(static_cast<unsigned short>(hv[v / 2] >> (16 * (v & 1))));
                }
            }
            if (divide && redo)
                corr_rows_exact<kVecW>(Ls, Rs, tw, RW, wl, rs, Cg, inv_cg, dd0, D, gx, W, zero_rule, op, plane);
        }
    }
}

// The same row streaming with an 8-column x 8-disparity register tile per
// thread (corr_volume_rows_kernel's is 4 x 8): per channel one 16-byte left
// load and two 16-byte right loads feed 64 fmas, and the epilogue stores 16
// bytes per disparity, so loads, epilogue and per-row overhead per output
// are about half.  Same arithmetic, so bit-identical results.  blockDim =
// (tw / 8, ny), DT = 8 ny.
template <int CC, int CG, int RULE>
__global__ void __maxnreg__(128) corr_volume_rows8_kernel(
    const __half* __restrict__ left, const __half* __restrict__ right, __half* __restrict__ out,
    int C, int H, int W, int D, int G, int rows, int tw, float inv_cg)
{
    constexpr int ND = kDispPerThread;
    constexpr int VW = 8;
    const int DT = ND * blockDim.y;
    const int RW = tw + DT;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __half* buf = reinterpret_cast<__half*>(smem_raw);
    const int buf_elems = CC * (tw + RW);

    const int w0 = blockIdx.x * tw;
    const int h0 = blockIdx.y * rows;
    const int h1 = min(h0 + rows, H);
    const int b = blockIdx.z / G;
    const int g = blockIdx.z - b * G;
    const int Cg = CG > 0 ? CG : C / G;
    const int64_t plane = i64(H) * W;
    const __half* lbase = left + (i64(b) * C + i64(g) * Cg) * plane;
    const __half* rbase = right + (i64(b) * C + i64(g) * Cg) * plane;

    const int wl = threadIdx.x * VW;
    const int dd0 = threadIdx.y * ND;
    const int rs = wl - dd0 - ND + DT;  // 8-aligned: right value k (0..15) is column wl - dd0 - 8 + k
    const int gx = w0 + wl;
    const bool full_cols = gx + VW <= W;
    constexpr bool divide = (RULE & kRuleDivide) != 0;  // as in corr_volume_rows_kernel
    constexpr bool zero_rule = (RULE & kRuleZero) != 0;
    const bool plain = dd0 + ND <= D && full_cols && !divide && !(zero_rule && gx < dd0 + ND - 1);
    __half* obase = out + ((i64(b) * G + g) * D + dd0) * plane + gx;

    auto stage = [&](int hh) {
        __half* nL = buf + ((hh - h0) % 3) * buf_elems;
        stage_rows_async(nL, lbase + i64(hh) * W, plane, Cg, w0, tw, W);
        stage_rows_async(nL + CC * tw, rbase + i64(hh) * W, plane, Cg, w0 - DT, RW, W);
    };
    if (h0 < h1) stage(h0);
    if (h0 + 1 < h1) stage(h0 + 1);
    for (int h = h0; h < h1; ++h) {
        const __half* Ls = buf + ((h - h0) % 3) * buf_elems;
        const __half* Rs = Ls + CC * tw;
        if (h + 1 < h1) asm volatile("cp.async.wait_group 2;\n" ::: "memory");
        else asm volatile("cp.async.wait_group 0;\n" ::: "memory");
        __syncthreads();  // row h landed for every thread; row h - 1's compute done everywhere
        if (h + 2 < h1) stage(h + 2);  // into row h - 1's buffer
        float acc[ND][VW];
#pragma unroll
        for (int i = 0; i < ND; ++i)
#pragma unroll
            for (int v = 0; v < VW; ++v) acc[i][v] = 0.0f;
#pragma unroll(CG > 0 ? CG : 1)
        for (int c = 0; c < Cg; ++c) {
            const uint4 l8 = *reinterpret_cast<const uint4*>(Ls + c * tw + wl);
            const __half* rp = Rs + c * RW + rs;
            const uint4 r0 = *reinterpret_cast<const uint4*>(rp);
            const uint4 r1 = *reinterpret_cast<const uint4*>(rp + 8);
            unsigned short lv[VW], rv[16];
            unpack_h2(l8.x, lv[0], lv[1]);
            unpack_h2(l8.y, lv[2], lv[3]);
            unpack_h2(l8.z, lv[4], lv[5]);
            unpack_h2(l8.w, lv[6], lv[7]);
            unpack_h2(r0.x, rv[0], rv[1]);
            unpack_h2(r0.y, rv[2], rv[3]);
            unpack_h2(r0.z, rv[4], rv[5]);
            unpack_h2(r0.w, rv[6], rv[7]);
            unpack_h2(r1.x, rv[8], rv[9]);
            unpack_h2(r1.y, rv[10], rv[11]);
            unpack_h2(r1.z, rv[12], rv[13]);
            unpack_h2(r1.w, rv[14], rv[15]);
#pragma unroll
            for (int dd = 0; dd < ND; ++dd)
#pragma unroll
                for (int v = 0; v < VW; ++v) acc[dd][v] = fma_h(lv[v], rv[ND - dd + v], acc[dd][v]);
        }
        __half* op = obase + i64(h) * W;
        if (plain) {
#pragma unroll
            for (int dd = 0; dd < ND; ++dd) {
                uint4 u;
                u.x = scale2_to_half2(acc[dd][0], acc[dd][1], inv_cg);
                u.y = scale2_to_half2(acc[dd][2], acc[dd][3], inv_cg);
                u.z = scale2_to_half2(acc[dd][4], acc[dd][5], inv_cg);
                u.w = scale2_to_half2(acc[dd][6], acc[dd][7], inv_cg);
                *reinterpret_cast<uint4*>(op + dd * plane) = u;
            }
        } else if (gx < W) {
            bool redo = false;  // as in corr_volume_rows_kernel
#pragma unroll
            for (int dd = 0; dd < ND; ++dd) {
                const int d = dd0 + dd;
                if (d >= D) break;
                uint32_t hv[VW / 2];
                redo |= scale_cols<VW, RULE>(acc[dd], gx, d, Cg, inv_cg, hv);
                __half* o = op + dd * plane;
                if (full_cols) {
                    *reinterpret_cast<uint4*>(o) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
                } else {
#pragma unroll
                    for (int v = 0; v < VW; ++v)
                        if (gx + v < W)
                            o[v] = __ushort_as_half(static_cast<unsigned short>(hv[v / 2] >> (16 * (v & 1))));
                }
            }
            if (divide && redo)
                corr_rows_exact<VW>(Ls, Rs, tw, RW, wl, rs, Cg, inv_cg, dd0, D, gx, W, zero_rule, op, plane);
        }
    }
}

// Small volumes (fewer than kSmallOutputsPerSM outputs per SM; the
// reference's native 1 x 48 x 32 x 40 is one): one thread per output, both
// operands read straight through L2, the channel loop unrolled so 8 channels'
// loads are in flight at once.  The tiled kernel gives such a volume a few
// dozen CTAs whose staging round trips and 2048-fma chains are latency the SMs
// cannot hide.  Same fp32 fma chain in channel order from +0, same scale rule
// and fp16 rounding, so the result is bit-identical to the tiled kernel's.
// Output index = ((((b G + g) D + d) H + h) W + w), the [B, G, D, H, W] layout.
template <typename T>
__global__ void __launch_bounds__(256) corr_volume_small_kernel(
    const T* __restrict__ left, const T* __restrict__ right, T* __restrict__ out,
    int C, int H, int W, int D, int G, int64_t total, int scale_div, float inv_cg)
{
    // total < sm_count * kSmallOutputsPerSM: 32-bit index arithmetic (64-bit
    // division is emulated and would cost more than the dot product).
    const int i = static_cast<int>(blockIdx.x) * 256 + static_cast<int>(threadIdx.x);
    if (i >= total) return;
    int r = i;
    const int w = r % W;
    r /= W;
    const int h = r % H;
    r /= H;
    const int d = r % D;
    r /= D;
    const int g = r % G;
    const int b = r / G;
    const int Cg = C / G;
    float val = 0.0f;  // w - d < 0: exact +0
    if (w >= d) {
        const int64_t plane = i64(H) * W;
        const int64_t base = (i64(b) * C + i64(g) * Cg) * plane + i64(h) * W;
        const T* lp = left + base + w;
        const T* rp = right + base + (w - d);
        float acc = 0.0f;
#pragma unroll 8
        for (int c = 0; c < Cg; ++c, lp += plane, rp += plane)
            acc = __fmaf_rn(to_f32<T>(__ldg(lp)), to_f32<T>(__ldg(rp)), acc);
        val = scale_div ? div_int(acc, Cg, inv_cg) : __fmul_rn(acc, inv_cg);
    }
    out[i] = from_f32<T>(val);
}

}  // namespace

namespace {

__device__ unsigned long long g_int_div_mismatch;

// div_int against the rounded division on every fp32 bit pattern a (NaN
// results compare equal to NaN).
__global__ void __launch_bounds__(256) int_div_selftest_kernel(int b, float y)
{
    unsigned long long bad = 0;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < (1ull << 32); i += stride) {
        const float a = __uint_as_float(static_cast<uint32_t>(i));
        const float q1 = div_int(a, b, y), q2 = __fdiv_rn(a, static_cast<float>(b));
        const bool same = __float_as_uint(q1) == __float_as_uint(q2) || (isnan(q1) && isnan(q2));
        bad += same ? 0u : 1u;
    }
    if (bad != 0) atomicAdd(&g_int_div_mismatch, bad);
}

}  // namespace

// Test hook: the number of fp32 values a for which div_int(a, b, RN(1/b))
// differs from the rounded division a / b (synchronises).
int int_div_selftest(int b, unsigned long long* mismatches) noexcept
{
    if (mismatches == nullptr) return WW_ERR_NULL_POINTER;
    if (b < 1 || b > kMaxIntDivisor) return WW_ERR_INVALID_SHAPE;
    DeviceInfo dev;
    if (current_device_info(&dev) != WW_SUCCESS) return WW_ERR_DEVICE;
    const unsigned long long zero = 0;
    if (cudaMemcpyToSymbol(g_int_div_mismatch, &zero, sizeof(zero)) != cudaSuccess) return launch_status("ww_selftest_int_division");
    int_div_selftest_kernel<<<dev.sm_count * 8, 256>>>(b, 1.0f / static_cast<float>(b));
    const int st = launch_status("ww_selftest_int_division");
    if (st != WW_SUCCESS) return st;
    if (cudaMemcpyFromSymbol(mismatches, g_int_div_mismatch, sizeof(*mismatches)) != cudaSuccess)
        return launch_status("ww_selftest_int_division");
    return WW_SUCCESS;
}

// The row-streaming kernel for a group width and scale rule (the width
// unrolled when it is 4, 8, 12 or 16; the rule always a template constant);
// eight: the 8 x 8 register tile, else the 4 x 8 one.
using RowsFn = void (*)(const __half*, const __half*, __half*, int, int, int, int, int, int, int, float);

template <int RULE>
RowsFn rows_kernel_for(int Cg, bool eight)
{
    if (eight)
        return Cg == 4    ? corr_volume_rows8_kernel<kChunkC, 4, RULE>
               : Cg == 8  ? corr_volume_rows8_kernel<kChunkC, 8, RULE>
               : Cg == 12 ? corr_volume_rows8_kernel<kChunkC, 12, RULE>
               : Cg == 16 ? corr_volume_rows8_kernel<kChunkC, 16, RULE>
                          : corr_volume_rows8_kernel<kChunkC, 0, RULE>;
    return Cg == 4    ? corr_volume_rows_kernel<kChunkC, 4, RULE>
           : Cg == 8  ? corr_volume_rows_kernel<kChunkC, 8, RULE>
           : Cg == 12 ? corr_volume_rows_kernel<kChunkC, 12, RULE>
           : Cg == 16 ? corr_volume_rows_kernel<kChunkC, 16, RULE>
                      : corr_volume_rows_kernel<kChunkC, 0, RULE>;
}

RowsFn rows_kernel(int Cg, int rule, bool eight)
{
    if (rule == 0) return rows_kernel_for<0>(Cg, eight);
    if (rule == kRuleZero) return rows_kernel_for<kRuleZero>(Cg, eight);
    return rows_kernel_for<kRuleZero | kRuleDivide>(Cg, eight);
}

// Scale rule of the reference kernel that launchCorrVolume<T> would run for a
// call with (B, C, H, W, D): 1 = naive kernel (acc / C), 0 = fast kernel
// (acc * 1/C).  Restates corr_volume_kernel.cu:251-326 (pickTileW and
// fastPathApplies) for the current device's SM count.
int corr_scale_div(bool is_half, int B, int C, int H, int W, int D, int sm_count) noexcept
{
    if (!is_half) return 1;                 // float always takes the naive kernel (:373)
    if (D <= 0 || D % 6 != 0) return 1;
    auto round_up = [](int v, int m) { return (v + m - 1) / m * m; };
    const int dispY = D / 6;
    const int PADA = round_up(D - 1, 8);
    // pickTileW
    int tile = round_up(W, 8);
    const int rowBlocks = H * B;
    const int target = sm_count / 2;
    if (rowBlocks > 0 && rowBlocks < target && tile > 64) {
        const int wantSplit = (target + rowBlocks - 1) / rowBlocks;
        const int split = round_up((W + wantSplit - 1) / wantSplit, 8);
        if (split > 0 && split < tile) tile = split;
        if (tile < 32) tile = 32;
    }
    const int byBytes = (48 * 1024 / (2 * C) - PADA) / 2;
    if (tile > byBytes) tile = byBytes;
    const int byThreads = 1024 / dispY * 4;
    if (tile > byThreads) tile = byThreads;
    tile = tile / 8 * 8;
    if (tile < 8) return 1;
    const int gridX = (W + tile - 1) / tile;
    if (gridX > 1) {
        const int balanced = round_up((W + gridX - 1) / gridX, 8);
        if (balanced >= 32 && balanced < tile) tile = balanced;
    }
    // fastPathApplies
    if (W % 8 != 0) return 1;
    if (static_cast<long long>(B) * D * H * W < static_cast<long long>(sm_count) * 800) return 1;
    if (tile < 8 || tile % 8 != 0) return 1;
    if (static_cast<long long>(C) * (2 * tile + PADA) * 2 > 48 * 1024) return 1;
    const int threads = (tile / 4) * dispY;
    if (threads <= 0 || threads > 1024) return 1;
    return 0;
}

// Group-wise scale rule: G == 1 is a single reference call over all C;
// G > 1 is the reference called once per (b, g) with B = 1, C = C/G.
int corr_scale_div_grouped(bool is_half, int B, int C, int G, int H, int W, int D, int sm_count) noexcept
{
    return G == 1 ? corr_scale_div(is_half, B, C, H, W, D, sm_count)
                  : corr_scale_div(is_half, 1, C / G, H, W, D, sm_count);
}

int corr_volume_launch(const void* left, const void* right, void* out, int dtype, int B, int C,
                       int H, int W, int D, int G, cudaStream_t stream) noexcept
{
    if (left == nullptr || right == nullptr || out == nullptr) return WW_ERR_NULL_POINTER;
    if (B < 0 || C <= 0 || H < 0 || W < 0 || D < 0 || G <= 0 || C % G != 0) return WW_ERR_INVALID_SHAPE;
    if (dtype != WW_DTYPE_HALF && dtype != WW_DTYPE_FLOAT) return WW_ERR_INVALID_DTYPE;
    if (B == 0 || H == 0 || W == 0 || D == 0) return WW_SUCCESS;
    if (static_cast<long long>(B) * G > 65535) return WW_ERR_UNSUPPORTED;
    DeviceInfo dev;
    if (current_device_info(&dev) != WW_SUCCESS) return WW_ERR_DEVICE;

    const bool is_half = dtype == WW_DTYPE_HALF;
    const int Cg = C / G;
    const int scale_div = corr_scale_div_grouped(is_half, B, C, G, H, W, D, dev.sm_count);
    const int rule = scale_div ? (kRuleZero | ((C / G) & (C / G - 1) ? kRuleDivide : 0)) : 0;
    const float inv_cg = 1.0f / static_cast<float>(Cg);

    const int64_t total = static_cast<int64_t>(B) * G * D * H * W;
    if (total < static_cast<int64_t>(dev.sm_count) * kSmallOutputsPerSM) {
        const unsigned blocks = static_cast<unsigned>((total + 255) / 256);
        if (is_half)
            corr_volume_small_kernel<__half><<<blocks, 256, 0, stream>>>(
                static_cast<const __half*>(left), static_cast<const __half*>(right), static_cast<__half*>(out),
                C, H, W, D, G, total, scale_div, inv_cg);
        else
            corr_volume_small_kernel<float><<<blocks, 256, 0, stream>>>(
                static_cast<const float*>(left), static_cast<const float*>(right), static_cast<float*>(out),
                C, H, W, D, G, total, scale_div, inv_cg);
        return launch_status("ww_corr_volume");
    }

    if (is_half && W > 64) {
        // Column tiles sized to the image: ceil(W / 256) tiles of up to 256
        // columns, a multiple of 16 (4 columns per thread).
        const int nt = (W + 255) / 256;
        const int tw = ((W + nt - 1) / nt + 15) / 16 * 16;
        const int tx = tw / kVecW;
        const int ny = max(1, min((D + kDispPerThread - 1) / kDispPerThread, 512 / tx));
        const int DT = ny * kDispPerThread;
        const int n_dband = (D + DT - 1) / DT;
        if (static_cast<long long>(H) * n_dband > 65535) return WW_ERR_UNSUPPORTED;
        const int cc = kChunkC;
        const size_t smem = static_cast<size_t>(cc) * (2 * tw + DT) * 2;
        const int vec_ok = (W % 8 == 0) && (reinterpret_cast<uintptr_t>(left) % 16 == 0) &&
                           (reinterpret_cast<uintptr_t>(right) % 16 == 0);
        // 8-column x 8-disparity tiles for groups of 8..16 channels and at
        // most 48 disparities (measured: configs 2 and 4 7 % and 3 % faster;
        // config 3 (D = 64, fewer resident warps at 121 registers) 23 % and
        // config 5 (Cg = 4) 11 % slower than the 4 x 8 tile).
        const int tx8 = tw / 8;
        const int ny8 = max(1, min((D + kDispPerThread - 1) / kDispPerThread, 512 / tx8));
        const int DT8 = ny8 * kDispPerThread;
        if (vec_ok && DT8 >= D && D <= 48 && Cg >= 8 && Cg <= cc) {
            const RowsFn kern = rows_kernel(Cg, rule, true);
            const size_t rsmem = 3 * static_cast<size_t>(cc) * (2 * tw + DT8) * 2;
            int resident = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, kern, tx8 * ny8, rsmem) != cudaSuccess ||
                resident < 1)
                return launch_status("ww_corr_volume");
            const long long slots = static_cast<long long>(resident) * dev.sm_count;
            const long long tiles = static_cast<long long>(nt) * B * G;
            int best = H;
            long long best_cost = -1;
            for (int r = 1; r <= H; ++r) {
                const long long ctas = tiles * ((H + r - 1) / r);
                const long long cost = ((ctas + slots - 1) / slots) * (r + 1);
                if (best_cost < 0 || cost < best_cost) { best_cost = cost; best = r; }
            }
            dim3 block(tx8, ny8);
            dim3 grid(nt, (H + best - 1) / best, B * G);
            kern<<<grid, block, rsmem, stream>>>(static_cast<const __half*>(left), static_cast<const __half*>(right),
                                                 static_cast<__half*>(out), C, H, W, D, G, best, tw, inv_cg);
            return launch_status("ww_corr_volume");
        }
        if (vec_ok && n_dband == 1 && Cg <= cc) {
            // Row-streaming form (two staged rows in shared memory): rows
            // per CTA chosen to minimise (waves of resident CTAs) x (rows
            // per CTA + 1 for the first row's copy).
            const size_t rsmem = 3 * smem;  // three staged rows
            const RowsFn kern = rows_kernel(Cg, rule, false);
            int resident = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, kern, tx * ny, rsmem) != cudaSuccess ||
                resident < 1)
                return launch_status("ww_corr_volume");
            const long long slots = static_cast<long long>(resident) * dev.sm_count;
            const long long tiles = static_cast<long long>(nt) * B * G;
            int best = H;
            long long best_cost = -1;
            for (int r = 1; r <= H; ++r) {
                const long long ctas = tiles * ((H + r - 1) / r);
                const long long cost = ((ctas + slots - 1) / slots) * (r + 1);
                if (best_cost < 0 || cost < best_cost) { best_cost = cost; best = r; }
            }
            dim3 block(tx, ny);
            dim3 grid(nt, (H + best - 1) / best, B * G);
            kern<<<grid, block, rsmem, stream>>>(
                static_cast<const __half*>(left), static_cast<const __half*>(right), static_cast<__half*>(out), C,
                H, W, D, G, best, tw, inv_cg);
            return launch_status("ww_corr_volume");
        }
        dim3 block(tx, ny);
        dim3 grid((W + tw - 1) / tw, H * n_dband, B * G);
        corr_volume_h_kernel<kChunkC><<<grid, block, smem, stream>>>(
            static_cast<const __half*>(left), static_cast<const __half*>(right), static_cast<__half*>(out), C, H, W,
            D, G, n_dband, tw, scale_div, inv_cg, vec_ok);
        return launch_status("ww_corr_volume");
    }

    // Tile shape: the narrowest column tile that covers a row (64 or 32 columns
    // = 16 or 8 threads across, 32-channel chunks) when the image is narrow:
    // the reference's native 32 x 40 would otherwise stage and compute three
    // times the columns it has.
    const int tw = W <= 32 ? 32 : (W <= 64 ? 64 : kTileW);
    // Narrow tiles keep 4 disparities per thread (twice the threads of the
    // 8 the wide tile keeps): a small image has few outputs, and the threads
    // are what hides the latency of its short fma chains.
    const int nd = tw == kTileW ? kDispPerThread : kDispPerThread / 2;
    int ny = min(tw == kTileW ? 8 : 16, (D + nd - 1) / nd);
    if (tw != kTileW) ny += ny & 1;  // DT a multiple of 8: the staged rows are 16-byte vectors
    const int DT = ny * nd;
    const int n_dband = (D + DT - 1) / DT;
    if (static_cast<long long>(H) * n_dband > 65535) return WW_ERR_UNSUPPORTED;
    dim3 block(tw / kVecW, ny);
    dim3 grid((W + tw - 1) / tw, H * n_dband, B * G);
    const size_t esize = is_half ? 2 : 4;
    const int cc = tw == kTileW ? kChunkC : 2 * kChunkC;
    const size_t smem = static_cast<size_t>(cc) * (tw + tw + DT) * esize;
    const int vec_elems = is_half ? 8 : 4;
    const int vec_ok = (W % vec_elems == 0) && (reinterpret_cast<uintptr_t>(left) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(right) % 16 == 0);
    auto launch = [&](auto tag) {
        using TT = decltype(tag);
        auto k = tw == 32 ? corr_volume_kernel<TT, 32, 2 * kChunkC>
                          : (tw == 64 ? corr_volume_kernel<TT, 64, 2 * kChunkC> : corr_volume_kernel<TT, kTileW, kChunkC>);
        k<<<grid, block, smem, stream>>>(static_cast<const TT*>(left), static_cast<const TT*>(right),
                                         static_cast<TT*>(out), C, H, W, D, G, n_dband, scale_div, inv_cg, vec_ok);
    };
    if (is_half) launch(__half{});
    else launch(float{});
    return launch_status("ww_corr_volume");
}

}  // namespace ww

// disparity_regression.cu -- soft-argmax / soft-argmin disparity regression
// over an aggregated cost volume, the step after the 3-D aggregation of a
// stereo network:
//
//   p[b, d, h, w]  = softmax_d( s * cost[b, d, h, w] ),  s = +1 (soft-argmax,
//                    cost is a similarity) or -1 (soft-argmin, cost is a
//                    matching cost)
//   disp[b, h, w]  = sum_d d * p[b, d, h, w]
//
// The reference library has no such op (its pipeline ends at the cost stem),
// so the op is specified here from the formula above; cost [B, D, H, W]
// (equivalently [B, 1, D, H, W]) fp16 or fp32, disparity [B, 1, H, W] fp16
// or fp32, fp32 arithmetic.
//
// B200 shape: the op reads every cost value once and writes one value per
// pixel, so it is HBM-bound (2 or 4 bytes per cost value); the exponentials
// are the only other cost (MUFU, 16 per SM per clock).  One pass over D with
// the softmax maximum updated per chunk of 8 disparities: the 8 values of a
// chunk are loaded together (8 independent loads in flight per thread),
// their maximum is taken, the running sums are rescaled once per chunk by
// 2^(M_old - M_new) and then take the 8 new terms 2^(x log2 e - M_new), where
// M = fp32(m log2 e) is the running maximum in log2 units as rounded: the
// exponent is formed by one fma (rounded once), and every term, old or new,
// is relative to the same rounded M, so M's rounding is a factor common to
// numerator and denominator and cancels (rescaling by the unrounded
// maximum instead would leave ~1e-4 relative error between chunks at
// |cost| ~ 1000).  A value costs one fma, one ex2 and one add -- not the two
// exponentials of a per-element online softmax.  A thread owns 4 horizontally adjacent pixels (8-byte fp16
// or 16-byte fp32 loads per disparity, 256 / 512 contiguous bytes per warp)
// when W is a multiple of 4 and the pointers are aligned, else 1 pixel.
#include "ww_common.cuh"

#include <cstdint>

namespace ww {
namespace {

constexpr int kChunk = 8;
constexpr int kBlock = 128;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float ex2_approx(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int VEC, typename Tin>
__device__ __forceinline__ void load_vec(const Tin* p, float (&v)[VEC]);

template <>
__device__ __forceinline__ void load_vec<4, __half>(const __half* p, float (&v)[4])
{
    const uint2 u = __ldcs(reinterpret_cast<const uint2*>(p));
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}

template <>
__device__ __forceinline__ void load_vec<4, float>(const float* p, float (&v)[4])
{
    const float4 u = __ldcs(reinterpret_cast<const float4*>(p));
    v[0] = u.x; v[1] = u.y; v[2] = u.z; v[3] = u.w;
}

template <>
__device__ __forceinline__ void load_vec<1, __half>(const __half* p, float (&v)[1])
{
    v[0] = __half2float(__ldcs(p));
}

template <>
__device__ __forceinline__ void load_vec<1, float>(const float* p, float (&v)[1])
{
    v[0] = __ldcs(p);
}

template <int VEC, typename Tout>
__device__ __forceinline__ void store_vec(Tout* p, const float (&v)[VEC]);

template <>
__device__ __forceinline__ void store_vec<4, __half>(__half* p, const float (&v)[4])
{
    const __half2 a = __floats2half2_rn(v[0], v[1]), b = __floats2half2_rn(v[2], v[3]);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&a);
    u.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = u;
}

template <>
__device__ __forceinline__ void store_vec<4, float>(float* p, const float (&v)[4])
{
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}

template <>
__device__ __forceinline__ void store_vec<1, __half>(__half* p, const float (&v)[1])
{
    *p = __float2half_rn(v[0]);
}

template <>
__device__ __forceinline__ void store_vec<1, float>(float* p, const float (&v)[1])
{
    *p = v[0];
}

struct DispParams {
    const void* cost;
    void* out;
    int D, H, W;
    int groups_w;      // pixel groups per image row (W / VEC)
    int64_t n_groups;  // B * H * groups_w
    float sign;        // +1 soft-argmax, -1 soft-argmin
};

// One thread per group of VEC pixels; the chunk loop keeps, per pixel, the
// running maximum M = fp32(m log2 e) of x = sign * cost, the softmax
// denominator s = sum 2^(x log2 e - M) and the numerator t = sum d * (...).
template <int VEC, typename Tin, typename Tout>
__global__ void __launch_bounds__(kBlock) disparity_regression_kernel(const DispParams p)
{
    const int64_t gid = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (gid >= p.n_groups) return;
    const int64_t per_image = static_cast<int64_t>(p.H) * p.groups_w;
    const int b = static_cast<int>(gid / per_image);
    const int64_t r = gid - static_cast<int64_t>(b) * per_image;
    const int h = static_cast<int>(r / p.groups_w);
    const int w0 = static_cast<int>(r - static_cast<int64_t>(h) * p.groups_w) * VEC;
    const int64_t plane = static_cast<int64_t>(p.H) * p.W;
    const Tin* src = static_cast<const Tin*>(p.cost) + static_cast<int64_t>(b) * p.D * plane +
                     static_cast<int64_t>(h) * p.W + w0;
    float m[VEC], s[VEC], t[VEC];
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
        m[k] = -INFINITY;
        s[k] = 0.0f;
        t[k] = 0.0f;
    }
    for (int d0 = 0; d0 < p.D; d0 += kChunk) {
        float x[kChunk][VEC];
#pragma unroll
        for (int j = 0; j < kChunk; ++j) {
            if (d0 + j < p.D) {
                load_vec<VEC, Tin>(src + static_cast<int64_t>(d0 + j) * plane, x[j]);
#pragma unroll
                for (int k = 0; k < VEC; ++k) x[j][k] *= p.sign;  // exact
            } else {
#pragma unroll
                for (int k = 0; k < VEC; ++k) x[j][k] = -INFINITY;
            }
        }
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
            float cm = x[0][k];
#pragma unroll
            for (int j = 1; j < kChunk; ++j) cm = fmaxf(cm, x[j][k]);
            const float mnl = fmaxf(m[k], cm * kLog2e);  // rounding is monotonic: fp32(max * log2 e)
            const float f = ex2_approx(m[k] - mnl);        // 0 on the first chunk (M = -inf)
            float sk = s[k] * f, tk = t[k] * f;
#pragma unroll
            for (int j = 0; j < kChunk; ++j) {
                const float e = ex2_approx(fmaf(x[j][k], kLog2e, -mnl));  // 0 for padded disparities
                sk += e;
                tk = fmaf(static_cast<float>(d0 + j), e, tk);
            }
            s[k] = sk;
            t[k] = tk;
            m[k] = mnl;
        }
    }
    float disp[VEC];
#pragma unroll
    for (int k = 0; k < VEC; ++k) disp[k] = __fdiv_rn(t[k], s[k]);
    Tout* dst = static_cast<Tout*>(p.out) + static_cast<int64_t>(b) * plane + static_cast<int64_t>(h) * p.W + w0;
    store_vec<VEC, Tout>(dst, disp);
}

// ---- packed fp32 pairs (sm_100 f32x2 arithmetic) ----
__device__ __forceinline__ uint64_t pk(float a, float b)
{
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void upk(uint64_t v, float& a, float& b)
{
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c)
{
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b)
{
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b)
{
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t h2f2(uint32_t h)
{
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
    return pk(f.x, f.y);
}
__device__ __forceinline__ uint64_t ex2_2(uint64_t v)
{
    float a, b;
    upk(v, a, b);
    return pk(ex2_approx(a), ex2_approx(b));
}

// The fp16-input, 4-pixel path with the same arithmetic per value as
// disparity_regression_kernel<4, __half, Tout> (same chunk maxima, the same
// fma exponent, the same order of the sums), in fewer instructions and
// registers: a chunk stays packed as 8 x (2 half2) = 16 registers, its
// maximum (minimum for soft-argmin, which is the maximum of -cost) is taken
// exactly on half2 pairs, and the exponent fma and both running sums run as
// f32x2 pairs.  Padded disparities load -inf (+inf for soft-argmin), whose
// exponent is -inf.
template <typename Tout, bool NEG>
__global__ void __launch_bounds__(kBlock) disparity_regression_h4_kernel(const DispParams p)
{
    const int64_t gid = static_cast<int64_t>(blockIdx.x) * kBlock + threadIdx.x;
    if (gid >= p.n_groups) return;
    const int64_t per_image = static_cast<int64_t>(p.H) * p.groups_w;
    const int b = static_cast<int>(gid / per_image);
    const int64_t r = gid - static_cast<int64_t>(b) * per_image;
    const int h = static_cast<int>(r / p.groups_w);
    const int w0 = static_cast<int>(r - static_cast<int64_t>(h) * p.groups_w) * 4;
    const int64_t plane = static_cast<int64_t>(p.H) * p.W;
    const __half* src = static_cast<const __half*>(p.cost) + static_cast<int64_t>(b) * p.D * plane +
                        static_cast<int64_t>(h) * p.W + w0;
    const float sl = NEG ? -kLog2e : kLog2e;
    const uint64_t sl2 = pk(sl, sl);
    const uint32_t pad = NEG ? 0x7C007C00u : 0xFC00FC00u;  // +inf / -inf half2
    float m[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    uint64_t s2[2] = {0, 0}, t2[2] = {0, 0};  // (+0, +0) pairs
    float fd0 = 0.0f;
    for (int d0 = 0; d0 < p.D; d0 += kChunk, fd0 += static_cast<float>(kChunk)) {
        uint2 raw[kChunk];
#pragma unroll
        for (int j = 0; j < kChunk; ++j)
            raw[j] = d0 + j < p.D ? __ldcs(reinterpret_cast<const uint2*>(src + static_cast<int64_t>(d0 + j) * plane))
                                  : make_uint2(pad, pad);
        __half2 c01 = *reinterpret_cast<const __half2*>(&raw[0].x);
        __half2 c23 = *reinterpret_cast<const __half2*>(&raw[0].y);
#pragma unroll
        for (int j = 1; j < kChunk; ++j) {
            const __half2 a = *reinterpret_cast<const __half2*>(&raw[j].x);
            const __half2 q = *reinterpret_cast<const __half2*>(&raw[j].y);
            c01 = NEG ? __hmin2(c01, a) : __hmax2(c01, a);
            c23 = NEG ? __hmin2(c23, q) : __hmax2(c23, q);
        }
        const float2 f01 = __half22float2(c01), f23 = __half22float2(c23);
        float mn[4] = {fmaxf(m[0], f01.x * sl), fmaxf(m[1], f01.y * sl), fmaxf(m[2], f23.x * sl),
                       fmaxf(m[3], f23.y * sl)};
        const uint64_t f2[2] = {pk(ex2_approx(m[0] - mn[0]), ex2_approx(m[1] - mn[1])),
                                pk(ex2_approx(m[2] - mn[2]), ex2_approx(m[3] - mn[3]))};
        const uint64_t nm2[2] = {pk(-mn[0], -mn[1]), pk(-mn[2], -mn[3])};
        s2[0] = mul2(s2[0], f2[0]);
        s2[1] = mul2(s2[1], f2[1]);
        t2[0] = mul2(t2[0], f2[0]);
        t2[1] = mul2(t2[1], f2[1]);
#pragma unroll
        for (int j = 0; j < kChunk; ++j) {
            const float dj = fd0 + static_cast<float>(j);  // exact; no int -> float conversion (XU pipe)
            const uint64_t d2 = pk(dj, dj);
            const uint64_t e01 = ex2_2(fma2(h2f2(raw[j].x), sl2, nm2[0]));
            const uint64_t e23 = ex2_2(fma2(h2f2(raw[j].y), sl2, nm2[1]));
            s2[0] = add2(s2[0], e01);
            s2[1] = add2(s2[1], e23);
            t2[0] = fma2(d2, e01, t2[0]);
            t2[1] = fma2(d2, e23, t2[1]);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) m[k] = mn[k];
    }
    float s[4], t[4];
    upk(s2[0], s[0], s[1]);
    upk(s2[1], s[2], s[3]);
    upk(t2[0], t[0], t[1]);
    upk(t2[1], t[2], t[3]);
    float disp[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) disp[k] = __fdiv_rn(t[k], s[k]);
    Tout* dst = static_cast<Tout*>(p.out) + static_cast<int64_t>(b) * plane + static_cast<int64_t>(h) * p.W + w0;
    store_vec<4, Tout>(dst, disp);
}

template <int VEC>
void launch_vec(const DispParams& p, int in_dtype, int out_dtype, cudaStream_t stream)
{
    const unsigned grid = static_cast<unsigned>((p.n_groups + kBlock - 1) / kBlock);
    const bool hi = in_dtype == WW_DTYPE_HALF, ho = out_dtype == WW_DTYPE_HALF;
    if (VEC == 4 && hi) {
        const bool neg = p.sign < 0.0f;
        if (ho && neg) disparity_regression_h4_kernel<__half, true><<<grid, kBlock, 0, stream>>>(p);
        else if (ho) disparity_regression_h4_kernel<__half, false><<<grid, kBlock, 0, stream>>>(p);
        else if (neg) disparity_regression_h4_kernel<float, true><<<grid, kBlock, 0, stream>>>(p);
        else disparity_regression_h4_kernel<float, false><<<grid, kBlock, 0, stream>>>(p);
        return;
    }
    if (hi && ho) disparity_regression_kernel<VEC, __half, __half><<<grid, kBlock, 0, stream>>>(p);
    else if (hi) disparity_regression_kernel<VEC, __half, float><<<grid, kBlock, 0, stream>>>(p);
    else if (ho) disparity_regression_kernel<VEC, float, __half><<<grid, kBlock, 0, stream>>>(p);
    else disparity_regression_kernel<VEC, float, float><<<grid, kBlock, 0, stream>>>(p);
}

}  // namespace

int disparity_regression_launch(const void* cost, void* out, int in_dtype, int out_dtype, int B, int D, int H,
                                int W, int mode, cudaStream_t stream) noexcept
{
    if (cost == nullptr || out == nullptr) return WW_ERR_NULL_POINTER;
    if ((in_dtype != WW_DTYPE_HALF && in_dtype != WW_DTYPE_FLOAT) ||
        (out_dtype != WW_DTYPE_HALF && out_dtype != WW_DTYPE_FLOAT))
        return WW_ERR_INVALID_DTYPE;
    if (mode != WW_DISP_SOFTARGMAX && mode != WW_DISP_SOFTARGMIN) return WW_ERR_UNSUPPORTED;
    if (B < 0 || D < 1 || H < 0 || W < 0) return WW_ERR_INVALID_SHAPE;
    if (B == 0 || H == 0 || W == 0) return WW_SUCCESS;
    DeviceInfo dev;
    if (current_device_info(&dev) != WW_SUCCESS) return WW_ERR_DEVICE;
    const int in_bytes = in_dtype == WW_DTYPE_HALF ? 2 : 4, out_bytes = out_dtype == WW_DTYPE_HALF ? 2 : 4;
    const bool vec = W % 4 == 0 && reinterpret_cast<uintptr_t>(cost) % (4 * in_bytes) == 0 &&
                     reinterpret_cast<uintptr_t>(out) % (4 * out_bytes) == 0;
    DispParams p;
    p.cost = cost;
    p.out = out;
    p.D = D;
    p.H = H;
    p.W = W;
    p.groups_w = vec ? W / 4 : W;
    p.n_groups = static_cast<int64_t>(B) * H * p.groups_w;
    p.sign = mode == WW_DISP_SOFTARGMIN ? -1.0f : 1.0f;
    if ((p.n_groups + kBlock - 1) / kBlock > 0x7fffffffLL) return WW_ERR_UNSUPPORTED;
    if (vec) launch_vec<4>(p, in_dtype, out_dtype, stream);
    else launch_vec<1>(p, in_dtype, out_dtype, stream);
    return launch_status("ww_disparity_regression");
}

}  // namespace ww

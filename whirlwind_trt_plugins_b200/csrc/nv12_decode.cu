// nv12_decode.cu -- NV12 -> normalised planar RGB (Nv12Decode) for B200:
// bilinear resize with align_corners = False and clamped taps, full-range
// BT.601 YCbCr -> RGB fused with 2 * (rgb / 255) - 1, fp16 or fp32 output,
// every batch item (the reference launcher, nv12_decode_kernel.cu:197-230,
// decodes one image; its plugin passes batch 0 only).
//
// Per pixel the arithmetic is the reference's (nv12_decode_kernel.cu:33-188)
// with the contractions nvcc applies to it written out as intrinsics, so the
// result does not depend on what the compiler contracts here:
//   src  = fma(dst + 0.5, scale, -0.5)
//   tap  = fma(w0, v0, w1 * v1) along x, then fma(wy0, top, wy1 * bottom)
//   R    = fma(2/255, fma(1.402, Cr, Y), -1)
//   G    = fma(2/255, fma(-0.714136, Cr, fma(-0.344136, Cb, Y)), -1)
//   B    = fma(2/255, fma(1.772, Cb, Y), -1),   Cb = U - 128, Cr = V - 128
//
// B200 shape: the op moves 1.5 bytes in per input pixel and 6 (fp16) or 12
// (fp32) bytes out per output pixel; nothing is reused beyond the 2x2 taps,
// which neighbouring outputs share through the read-only cache; a chroma tap
// is one 2-byte load of its (U, V) pair (8 loads per output pixel rather than
// 12: the launch is bound by load latency and issue, not bandwidth).  One thread
// makes two horizontally adjacent output pixels, so a warp writes 128-byte
// (fp16) or 256-byte (fp32) contiguous runs of each colour plane with one
// vector store per lane.  Grid (ceil(W_OUT / 64), ceil(H_OUT / 8), B) of
// 32 x 8 threads.
#include "ww_common.cuh"

#include <cstdint>

namespace ww {
namespace {

constexpr int kBx = 32, kBy = 8, kPix = 2;

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// Bilinear tap of an 8-bit plane: `step` bytes between horizontal samples
// (1 for Y, 2 for the interleaved chroma), `stride` bytes per row.
__device__ __forceinline__ float bilinear(const uint8_t* __restrict__ plane, int rows, int cols, int stride,
                                          int step, float yf, float xf)
{
    const float fy = floorf(yf), fx = floorf(xf);
    const int y0 = static_cast<int>(fy), x0 = static_cast<int>(fx);
    const float wy1 = __fsub_rn(yf, fy), wy0 = __fsub_rn(1.0f, wy1);
    const float wx1 = __fsub_rn(xf, fx), wx0 = __fsub_rn(1.0f, wx1);
    const int y0c = clampi(y0, 0, rows - 1), y1c = clampi(y0 + 1, 0, rows - 1);
    const int x0c = clampi(x0, 0, cols - 1) * step, x1c = clampi(x0 + 1, 0, cols - 1) * step;
    const uint8_t* r0 = plane + static_cast<int64_t>(y0c) * stride;
    const uint8_t* r1 = plane + static_cast<int64_t>(y1c) * stride;
    const float v00 = static_cast<float>(__ldg(r0 + x0c)), v01 = static_cast<float>(__ldg(r0 + x1c));
    const float v10 = static_cast<float>(__ldg(r1 + x0c)), v11 = static_cast<float>(__ldg(r1 + x1c));
    const float top = __fmaf_rn(wx0, v00, __fmul_rn(wx1, v01));
    const float bot = __fmaf_rn(wx0, v10, __fmul_rn(wx1, v11));
    return __fmaf_rn(wy0, top, __fmul_rn(wy1, bot));
}

// Both chroma channels of one tap position at once: U and V are adjacent
// bytes, so each of the four taps is one 2-byte load, and the weights and
// clamped indices are computed once.  Per channel the arithmetic is that of
// bilinear(plane, rows, cols, stride, 2, yf, xf) (and of it at plane + 1).
__device__ __forceinline__ void bilinear_uv(const uint8_t* __restrict__ chroma, int rows, int cols, int stride,
                                            float yf, float xf, float& u, float& v)
{
    const float fy = floorf(yf), fx = floorf(xf);
    const int y0 = static_cast<int>(fy), x0 = static_cast<int>(fx);
    const float wy1 = __fsub_rn(yf, fy), wy0 = __fsub_rn(1.0f, wy1);
    const float wx1 = __fsub_rn(xf, fx), wx0 = __fsub_rn(1.0f, wx1);
    const int y0c = clampi(y0, 0, rows - 1), y1c = clampi(y0 + 1, 0, rows - 1);
    const int x0c = clampi(x0, 0, cols - 1) * 2, x1c = clampi(x0 + 1, 0, cols - 1) * 2;
    const uint8_t* r0 = chroma + static_cast<int64_t>(y0c) * stride;
    const uint8_t* r1 = chroma + static_cast<int64_t>(y1c) * stride;
    // even byte offsets from an even base (the chroma plane starts at
    // H_IN * W_IN and W_IN is even): 2-byte aligned; low byte U, high byte V
    const unsigned short t00 = __ldg(reinterpret_cast<const unsigned short*>(r0 + x0c));
    const unsigned short t01 = __ldg(reinterpret_cast<const unsigned short*>(r0 + x1c));
    const unsigned short t10 = __ldg(reinterpret_cast<const unsigned short*>(r1 + x0c));
    const unsigned short t11 = __ldg(reinterpret_cast<const unsigned short*>(r1 + x1c));
    auto lerp = [&](int sh) {
        const float v00 = static_cast<float>((t00 >> sh) & 0xff), v01 = static_cast<float>((t01 >> sh) & 0xff);
        const float v10 = static_cast<float>((t10 >> sh) & 0xff), v11 = static_cast<float>((t11 >> sh) & 0xff);
        const float top = __fmaf_rn(wx0, v00, __fmul_rn(wx1, v01));
        const float bot = __fmaf_rn(wx0, v10, __fmul_rn(wx1, v11));
        return __fmaf_rn(wy0, top, __fmul_rn(wy1, bot));
    };
    u = lerp(0);
    v = lerp(8);
}

struct Nv12Params {
    const uint8_t* nv12;
    void* out;
    int H_IN, W_IN, H_OUT, W_OUT;
    float sy_h, sy_w, suv_h, suv_w;
    int vec;       // 1: W_OUT even and the output 8-byte aligned (paired stores)
    int uv_pairs;  // 1: W_IN even and the input 2-byte aligned (one load per chroma tap)
};

template <bool F16>
__global__ void __launch_bounds__(kBx * kBy) nv12_decode_kernel(const Nv12Params p)
{
    const int x0 = (blockIdx.x * kBx + threadIdx.x) * kPix;
    const int y = blockIdx.y * kBy + threadIdx.y;
    const int b = blockIdx.z;
    if (y >= p.H_OUT || x0 >= p.W_OUT) return;
    const int64_t in_img = static_cast<int64_t>(p.H_IN * 3 / 2) * p.W_IN;
    const uint8_t* img = p.nv12 + b * in_img;
    const uint8_t* chroma = img + static_cast<int64_t>(p.H_IN) * p.W_IN;
    const int H_UV = p.H_IN >> 1, W_UV = p.W_IN >> 1;
    constexpr float s = 2.0f / 255.0f;

    const float yf_y = __fmaf_rn(__fadd_rn(static_cast<float>(y), 0.5f), p.sy_h, -0.5f);
    const float yf_uv = __fmaf_rn(__fadd_rn(static_cast<float>(y), 0.5f), p.suv_h, -0.5f);
    float rgb[3][kPix];
#pragma unroll
    for (int j = 0; j < kPix; ++j) {
        const float xo = __fadd_rn(static_cast<float>(x0 + j), 0.5f);
        const float xf_y = __fmaf_rn(xo, p.sy_w, -0.5f);
        const float xf_uv = __fmaf_rn(xo, p.suv_w, -0.5f);
        const float Y = bilinear(img, p.H_IN, p.W_IN, p.W_IN, 1, yf_y, xf_y);
        float U, V;
        if (p.uv_pairs) {
            bilinear_uv(chroma, H_UV, W_UV, p.W_IN, yf_uv, xf_uv, U, V);
        } else {
            U = bilinear(chroma, H_UV, W_UV, p.W_IN, 2, yf_uv, xf_uv);
            V = bilinear(chroma + 1, H_UV, W_UV, p.W_IN, 2, yf_uv, xf_uv);
        }
        const float Cb = __fsub_rn(U, 128.0f), Cr = __fsub_rn(V, 128.0f);
        rgb[0][j] = __fmaf_rn(s, __fmaf_rn(1.402f, Cr, Y), -1.0f);
        rgb[1][j] = __fmaf_rn(s, __fmaf_rn(-0.714136f, Cr, __fmaf_rn(-0.344136f, Cb, Y)), -1.0f);
        rgb[2][j] = __fmaf_rn(s, __fmaf_rn(1.772f, Cb, Y), -1.0f);
    }

    const int64_t plane = static_cast<int64_t>(p.H_OUT) * p.W_OUT;
    const int64_t o = b * 3 * plane + static_cast<int64_t>(y) * p.W_OUT + x0;
    const bool pair = p.vec != 0;  // then x0 + 1 < W_OUT as well (W_OUT even)
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        if constexpr (F16) {
            __half* dst = static_cast<__half*>(p.out) + o + c * plane;
            if (pair) {
                *reinterpret_cast<__half2*>(dst) = __floats2half2_rn(rgb[c][0], rgb[c][1]);
            } else {
                dst[0] = __float2half_rn(rgb[c][0]);
                if (x0 + 1 < p.W_OUT) dst[1] = __float2half_rn(rgb[c][1]);
            }
        } else {
            float* dst = static_cast<float*>(p.out) + o + c * plane;
            if (pair) {
                *reinterpret_cast<float2*>(dst) = make_float2(rgb[c][0], rgb[c][1]);
            } else {
                dst[0] = rgb[c][0];
                if (x0 + 1 < p.W_OUT) dst[1] = rgb[c][1];
            }
        }
    }
}

}  // namespace

int nv12_decode_launch(const void* nv12, void* out, int dtype, int B, int H_IN, int W_IN, int H_OUT, int W_OUT,
                       cudaStream_t stream) noexcept
{
    if (nv12 == nullptr || out == nullptr) return WW_ERR_NULL_POINTER;
    if (dtype != WW_DTYPE_HALF && dtype != WW_DTYPE_FLOAT) return WW_ERR_INVALID_DTYPE;
    if (B < 0 || H_IN < 2 || W_IN < 2 || H_OUT < 1 || W_OUT < 1) return WW_ERR_INVALID_SHAPE;
    if (B == 0) return WW_SUCCESS;
    const int gx = (W_OUT + kBx * kPix - 1) / (kBx * kPix), gy = (H_OUT + kBy - 1) / kBy;
    if (B > 65535 || gy > 65535) return WW_ERR_UNSUPPORTED;
    DeviceInfo dev;
    if (current_device_info(&dev) != WW_SUCCESS) return WW_ERR_DEVICE;
    Nv12Params p;
    p.nv12 = static_cast<const uint8_t*>(nv12);
    p.out = out;
    p.H_IN = H_IN;
    p.W_IN = W_IN;
    p.H_OUT = H_OUT;
    p.W_OUT = W_OUT;
    // nv12_decode_kernel.cu:213-216
    p.sy_h = static_cast<float>(H_IN) / static_cast<float>(H_OUT);
    p.sy_w = static_cast<float>(W_IN) / static_cast<float>(W_OUT);
    p.suv_h = static_cast<float>(H_IN >> 1) / static_cast<float>(H_OUT);
    p.suv_w = static_cast<float>(W_IN >> 1) / static_cast<float>(W_OUT);
    p.vec = (W_OUT % 2 == 0) && (reinterpret_cast<uintptr_t>(out) % 8 == 0);
    p.uv_pairs = (W_IN % 2 == 0) && (reinterpret_cast<uintptr_t>(nv12) % 2 == 0);
    const dim3 grid(gx, gy, B), block(kBx, kBy);
    if (dtype == WW_DTYPE_HALF) nv12_decode_kernel<true><<<grid, block, 0, stream>>>(p);
    else nv12_decode_kernel<false><<<grid, block, 0, stream>>>(p);
    return launch_status("ww_nv12_decode");
}

}  // namespace ww

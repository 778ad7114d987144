// cost_stem3d_ref3.cu -- the reference's 7-input CostStem3D for B200:
// three Conv3d 3x3x3 pad 1 (1 -> 4 -> 4 -> 1) + folded-BN bias + ReLU6, fp16
// between stages (cost_stem_3d_kernel.cu:71-233), for every batch item.
//
// Per output value the arithmetic is the reference's, operation for
// operation: an fp32 fma chain in (ci, kd, kh, kw) order starting from +0,
// then + bias, ReLU6, round to fp16; intermediate positions outside the
// volume are exactly 0 for the next stage.  The result is bit-identical to
// the reference kernel whatever the tiling, so the tiling is B200's own:
//
//   * one CTA = a 4 x 8 x 8 (D, H, W) output brick of one batch item, 256
//     threads, one output per thread in the last stage;
//   * the input brick (+3 halo) and both intermediate bricks live in shared
//     memory as fp32 copies of fp16 values (no conversion in the inner loops),
//     36 KB, so six CTAs fit an SM;
//   * weights and biases are staged once per CTA into shared memory as fp32.
// The native shape [1, 1, 48, 32, 40] is launch-bound (~60K outputs): the
// grid is 240 CTAs, all resident in one wave on 148 SMs.

#include "ww_common.cuh"

namespace ww {
namespace {

constexpr int TD = 4, TH = 8, TW = 8;
constexpr int I_D = TD + 6, I_H = TH + 6, I_W = TW + 6;   // input brick
constexpr int A_D = TD + 4, A_H = TH + 4, A_W = TW + 4;   // stage-0 brick
constexpr int B_D = TD + 2, B_H = TH + 2, B_W = TW + 2;   // stage-1 brick
constexpr int I_VOL = I_D * I_H * I_W;
constexpr int A_VOL = A_D * A_H * A_W;
constexpr int B_VOL = B_D * B_H * B_W;
constexpr int kThreads = TD * TH * TW;  // 256
constexpr int kWeights = 108 + 4 + 432 + 4 + 108 + 1;

__device__ __forceinline__ float relu6(float v) { return fminf(6.0f, fmaxf(0.0f, v)); }

__device__ __forceinline__ bool inside(int d, int h, int w, int D, int H, int W)
{
    return d >= 0 && d < D && h >= 0 && h < H && w >= 0 && w < W;
}

__global__ void __launch_bounds__(kThreads) cost_stem3d_ref3_kernel(
    const __half* __restrict__ in, __half* __restrict__ out,
    const __half* __restrict__ w0, const __half* __restrict__ b0,
    const __half* __restrict__ w1, const __half* __restrict__ b1,
    const __half* __restrict__ w2, const __half* __restrict__ b2,
    int D, int H, int W, int n_dtiles)
{
    __shared__ float s_in[I_VOL];
    __shared__ float s_a[4 * A_VOL];
    __shared__ float s_b[4 * B_VOL];
    __shared__ float s_w[kWeights];
    float* sw0 = s_w;
    float* sb0 = sw0 + 108;
    float* sw1 = sb0 + 4;
    float* sb1 = sw1 + 432;
    float* sw2 = sb1 + 4;
    float* sb2 = sw2 + 108;

    const int tid = threadIdx.x;
    const int b = blockIdx.z / n_dtiles;
    const int od0 = (blockIdx.z - b * n_dtiles) * TD;
    const int oh0 = blockIdx.y * TH;
    const int ow0 = blockIdx.x * TW;
    const int64_t vol = i64(D) * H * W;
    const __half* src = in + i64(b) * vol;

    for (int i = tid; i < kWeights; i += kThreads) {
        float v;
        if (i < 108) v = __half2float(w0[i]);
        else if (i < 112) v = __half2float(b0[i - 108]);
        else if (i < 544) v = __half2float(w1[i - 112]);
        else if (i < 548) v = __half2float(b1[i - 544]);
        else if (i < 656) v = __half2float(w2[i - 548]);
        else v = __half2float(b2[0]);
        s_w[i] = v;
    }
    // Input brick, origin (od0-3, oh0-3, ow0-3), zero outside the volume.
    for (int i = tid; i < I_VOL; i += kThreads) {
        const int z = i / (I_H * I_W), r = i - z * I_H * I_W, y = r / I_W, x = r - y * I_W;
        const int gd = od0 - 3 + z, gh = oh0 - 3 + y, gw = ow0 - 3 + x;
        s_in[i] = inside(gd, gh, gw, D, H, W) ? __half2float(src[(i64(gd) * H + gh) * W + gw]) : 0.0f;
    }
    __syncthreads();

    // Stage 0: 1 -> 4 over the stage-0 brick, origin (od0-2, oh0-2, ow0-2).
    for (int i = tid; i < 4 * A_VOL; i += kThreads) {
        const int co = i / A_VOL, r0 = i - co * A_VOL;
        const int z = r0 / (A_H * A_W), r = r0 - z * A_H * A_W, y = r / A_W, x = r - y * A_W;
        float acc = 0.0f;
#pragma unroll
        for (int kd = 0; kd < 3; ++kd)
#pragma unroll
            for (int kh = 0; kh < 3; ++kh)
#pragma unroll
                for (int kw = 0; kw < 3; ++kw)
                    acc = __fmaf_rn(s_in[((z + kd) * I_H + y + kh) * I_W + x + kw], sw0[co * 27 + kd * 9 + kh * 3 + kw], acc);
        acc = __fadd_rn(acc, sb0[co]);
        const bool in_vol = inside(od0 - 2 + z, oh0 - 2 + y, ow0 - 2 + x, D, H, W);
        s_a[i] = in_vol ? __half2float(__float2half_rn(relu6(acc))) : 0.0f;
    }
    __syncthreads();

    // Stage 1: 4 -> 4 over the stage-1 brick, origin (od0-1, oh0-1, ow0-1).
    for (int i = tid; i < 4 * B_VOL; i += kThreads) {
        const int co = i / B_VOL, r0 = i - co * B_VOL;
        const int z = r0 / (B_H * B_W), r = r0 - z * B_H * B_W, y = r / B_W, x = r - y * B_W;
        float acc = 0.0f;
#pragma unroll
        for (int ci = 0; ci < 4; ++ci)
#pragma unroll
            for (int kd = 0; kd < 3; ++kd)
#pragma unroll
                for (int kh = 0; kh < 3; ++kh)
#pragma unroll
                    for (int kw = 0; kw < 3; ++kw)
                        acc = __fmaf_rn(s_a[ci * A_VOL + ((z + kd) * A_H + y + kh) * A_W + x + kw],
                                        sw1[(co * 4 + ci) * 27 + kd * 9 + kh * 3 + kw], acc);
        acc = __fadd_rn(acc, sb1[co]);
        const bool in_vol = inside(od0 - 1 + z, oh0 - 1 + y, ow0 - 1 + x, D, H, W);
        s_b[i] = in_vol ? __half2float(__float2half_rn(relu6(acc))) : 0.0f;
    }
    __syncthreads();

    // Stage 2: 4 -> 1, one output per thread.
    {
        const int z = tid / (TH * TW), r = tid - z * TH * TW, y = r / TW, x = r - y * TW;
        const int gd = od0 + z, gh = oh0 + y, gw = ow0 + x;
        if (gd < D && gh < H && gw < W) {
            float acc = 0.0f;
#pragma unroll
            for (int ci = 0; ci < 4; ++ci)
#pragma unroll
                for (int kd = 0; kd < 3; ++kd)
#pragma unroll
                    for (int kh = 0; kh < 3; ++kh)
#pragma unroll
                        for (int kw = 0; kw < 3; ++kw)
                            acc = __fmaf_rn(s_b[ci * B_VOL + ((z + kd) * B_H + y + kh) * B_W + x + kw],
                                            sw2[ci * 27 + kd * 9 + kh * 3 + kw], acc);
            acc = __fadd_rn(acc, sb2[0]);
            out[i64(b) * vol + (i64(gd) * H + gh) * W + gw] = __float2half_rn(relu6(acc));
        }
    }
}

}  // namespace

int cost_stem3d_ref3_launch(const void* in, void* out, const void* w0, const void* b0,
                            const void* w1, const void* b1, const void* w2, const void* b2,
                            int B, int D, int H, int W, cudaStream_t stream) noexcept
{
    if (!in || !out || !w0 || !b0 || !w1 || !b1 || !w2 || !b2) return WW_ERR_NULL_POINTER;
    if (B < 0 || D < 0 || H < 0 || W < 0) return WW_ERR_INVALID_SHAPE;
    if (B == 0 || D == 0 || H == 0 || W == 0) return WW_SUCCESS;
    const int n_dtiles = (D + TD - 1) / TD;
    if (static_cast<long long>(B) * n_dtiles > 65535 || (H + TH - 1) / TH > 65535) return WW_ERR_UNSUPPORTED;
    DeviceInfo dev;
    if (current_device_info(&dev) != WW_SUCCESS) return WW_ERR_DEVICE;
    dim3 grid((W + TW - 1) / TW, (H + TH - 1) / TH, B * n_dtiles);
    auto h = [](const void* p) { return static_cast<const __half*>(p); };
    cost_stem3d_ref3_kernel<<<grid, kThreads, 0, stream>>>(h(in), static_cast<__half*>(out), h(w0), h(b0),
                                                           h(w1), h(b1), h(w2), h(b2), D, H, W, n_dtiles);
    return launch_status("ww_cost_stem3d_ref3");
}

}  // namespace ww

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
//     threads;
//   * the input brick (+3 halo) and both intermediate bricks live in shared
//     memory as fp32 copies of fp16 values (no conversion in the inner loops),
//     36 KB, so six CTAs fit an SM;
//   * weights and biases are staged once per CTA into shared memory as fp32;
//   * each thread computes a run of NX consecutive outputs of one channel
//     (conv_run): NX independent fma chains advance together, one row segment
//     of NX + 2 inputs is loaded per (ci, kd, kh) and reused by the three kw
//     taps.  Each chain still runs in (ci, kd, kh, kw) order.
// The native shape [1, 1, 48, 32, 40] is latency-bound (~60K outputs, 240
// CTAs in one wave on 148 SMs): the independent chains are what hides the
// fma and shared-memory latency.

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

// NX consecutive outputs (x0 .. x0 + NX - 1, row y, plane z of the output
// brick) of one output channel of a 3x3x3 convolution over CIN channels of a
// shared-memory brick (channel stride cs, plane SH x SW).  w: [CIN][27].
template <int CIN, int NX>
__device__ __forceinline__ void conv_run(const float* src, int cs, int SH, int SW, int z, int y, int x0,
                                         const float* w, float (&acc)[NX])
{
#pragma unroll
    for (int j = 0; j < NX; ++j) acc[j] = 0.0f;
#pragma unroll
    for (int ci = 0; ci < CIN; ++ci)
#pragma unroll
        for (int kd = 0; kd < 3; ++kd)
#pragma unroll
            for (int kh = 0; kh < 3; ++kh) {
                const float* row = src + ci * cs + ((z + kd) * SH + y + kh) * SW + x0;
                float seg[NX + 2];
#pragma unroll
                for (int t = 0; t < NX + 2; ++t) seg[t] = row[t];
#pragma unroll
                for (int kw = 0; kw < 3; ++kw) {
                    const float wv = w[ci * 27 + kd * 9 + kh * 3 + kw];
#pragma unroll
                    for (int j = 0; j < NX; ++j) acc[j] = __fmaf_rn(seg[j + kw], wv, acc[j]);
                }
            }
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

    // Stage 0: 1 -> 4 over the stage-0 brick, origin (od0-2, oh0-2, ow0-2);
    // runs of 4 along the 12-wide rows.
    {
        constexpr int NX = 4, NG = A_W / NX;
        for (int i = tid; i < 4 * A_D * A_H * NG; i += kThreads) {
            const int co = i / (A_D * A_H * NG), r0 = i - co * (A_D * A_H * NG);
            const int z = r0 / (A_H * NG), r = r0 - z * (A_H * NG), y = r / NG, x0 = (r - y * NG) * NX;
            float acc[NX];
            conv_run<1, NX>(s_in, 0, I_H, I_W, z, y, x0, sw0 + co * 27, acc);
#pragma unroll
            for (int j = 0; j < NX; ++j) {
                const float v = __fadd_rn(acc[j], sb0[co]);
                const bool in_vol = inside(od0 - 2 + z, oh0 - 2 + y, ow0 - 2 + x0 + j, D, H, W);
                s_a[co * A_VOL + (z * A_H + y) * A_W + x0 + j] = in_vol ? __half2float(__float2half_rn(relu6(v))) : 0.0f;
            }
        }
    }
    __syncthreads();

    // Stage 1: 4 -> 4 over the stage-1 brick, origin (od0-1, oh0-1, ow0-1);
    // runs of 5 along the 10-wide rows.
    {
        constexpr int NX = 5, NG = B_W / NX;
        for (int i = tid; i < 4 * B_D * B_H * NG; i += kThreads) {
            const int co = i / (B_D * B_H * NG), r0 = i - co * (B_D * B_H * NG);
            const int z = r0 / (B_H * NG), r = r0 - z * (B_H * NG), y = r / NG, x0 = (r - y * NG) * NX;
            float acc[NX];
            conv_run<4, NX>(s_a, A_VOL, A_H, A_W, z, y, x0, sw1 + co * 108, acc);
#pragma unroll
            for (int j = 0; j < NX; ++j) {
                const float v = __fadd_rn(acc[j], sb1[co]);
                const bool in_vol = inside(od0 - 1 + z, oh0 - 1 + y, ow0 - 1 + x0 + j, D, H, W);
                s_b[co * B_VOL + (z * B_H + y) * B_W + x0 + j] = in_vol ? __half2float(__float2half_rn(relu6(v))) : 0.0f;
            }
        }
    }
    __syncthreads();

    // Stage 2: 4 -> 1, runs of 2 along the 8-wide output rows.
    {
        constexpr int NX = 2, NG = TW / NX;
        if (tid < TD * TH * NG) {
            const int z = tid / (TH * NG), r = tid - z * (TH * NG), y = r / NG, x0 = (r - y * NG) * NX;
            float acc[NX];
            conv_run<4, NX>(s_b, B_VOL, B_H, B_W, z, y, x0, sw2, acc);
            const int gd = od0 + z, gh = oh0 + y;
#pragma unroll
            for (int j = 0; j < NX; ++j) {
                const int gw = ow0 + x0 + j;
                if (gd < D && gh < H && gw < W)
                    out[i64(b) * vol + (i64(gd) * H + gh) * W + gw] =
                        __float2half_rn(relu6(__fadd_rn(acc[j], sb2[0])));
            }
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

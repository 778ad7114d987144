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
//   * weights and biases are staged once per CTA into shared memory as fp32,
//     the 4-output stages' weights as one float4 (the 4 output channels) per
//     (input channel, tap);
//   * in the two 4-output stages each thread computes a run of NX
//     consecutive positions for all 4 output channels (conv_run_x4): one row
//     segment of NX + 2 inputs is loaded per (ci, kd, kh) and reused by the
//     three kw taps and the four output channels, so a row costs NX + 2
//     scalar loads and 3 broadcast float4 loads for 12 NX fmas; the last
//     stage (one output channel) blocks 2 rows x 2 columns per thread;
//   * every global load of the staging phase is issued before the first
//     shared-memory store, so the brick costs one memory latency, not eight.
// Shared-memory bandwidth, not the fma rate, bounded the first version of
// this kernel (one output channel per thread, one weight load per tap).
// The native shape [1, 1, 48, 32, 40] is latency-bound (~60K outputs, 240
// CTAs in one wave on 148 SMs): the 4 NX independent chains per thread are
// what hides the fma and shared-memory latency.

#include "int_div.cuh"
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

// NX consecutive positions (x0 .. x0 + NX - 1, row y, plane z of the
// destination brick) of all 4 output channels of a 3x3x3 convolution over CIN
// channels of a shared-memory brick (channel stride cs, plane SH x SW).
// wq: [CIN][27] float4, one lane per output channel.  Each acc[co][j] is an
// fp32 fma chain in (ci, kd, kh, kw) order starting from +0.
template <int CIN, int NX>
__device__ __forceinline__ void conv_run_x4(const float* src, int cs, int SH, int SW, int z, int y, int x0,
                                            const float4* wq, float (&acc)[4][NX])
{
#pragma unroll
    for (int co = 0; co < 4; ++co)
#pragma unroll
        for (int j = 0; j < NX; ++j) acc[co][j] = 0.0f;
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
                    const float4 wv = wq[ci * 27 + kd * 9 + kh * 3 + kw];
#pragma unroll
                    for (int j = 0; j < NX; ++j) {
                        acc[0][j] = __fmaf_rn(seg[j + kw], wv.x, acc[0][j]);
                        acc[1][j] = __fmaf_rn(seg[j + kw], wv.y, acc[1][j]);
                        acc[2][j] = __fmaf_rn(seg[j + kw], wv.z, acc[2][j]);
                        acc[3][j] = __fmaf_rn(seg[j + kw], wv.w, acc[3][j]);
                    }
                }
            }
}

struct Ref3Params {
    const __half* in;     // stem input [B, 1, D, H, W] (CORR = false)
    const __half* left;   // features [B, C, H, W] (CORR = true)
    const __half* right;
    __half* out;          // [B, 1, D, H, W]
    const __half *w0, *b0, *w1, *b1, *w2, *b2;
    int C, D, H, W, n_dtiles;
    int scale_div;        // correlation scale rule: 1 acc / C, 0 acc * (1 / C)
    float inv_c;
    int vec_ok;           // W % 8 == 0 and 16-byte aligned features: vector segment loads
};

// Correlation staging (CORR = true): per chunk of kCorrC channels, fp16, in
// the space of the two intermediate bricks (free until stage 0), as 16-byte
// segments aligned in the image row: the left rows [c][14][24 columns from
// ow0 - 8] (the brick needs ow0 - 3 .. ow0 + 10) and the right rows
// [c][14][32 columns from rw0 rounded down to 8] (the brick needs
// rw0 = ow0 - od0 - 9 .. rw0 + 22, every w - d it holds).  A thread issues
// all kStageIt of its segment loads of a chunk before it stores any (one
// memory latency per chunk).
constexpr int kCorrC = 16;
constexpr int kLW = 24, kRWs = 32;            // staged columns per row
constexpr int kLSeg = I_H * kLW / 8;          // 42 segments per channel
constexpr int kRSeg = I_H * kRWs / 8;         // 56
constexpr int kSegC = kLSeg + kRSeg;          // 98
constexpr int kStageIt = (kCorrC * kSegC + kThreads - 1) / kThreads;
constexpr int kLTile = I_H * I_W;             // 196 brick positions (y, x)
static_assert(kCorrC * kSegC * 16 <= (4 * A_VOL + 4 * B_VOL) * 4, "correlation tiles exceed the brick space");
static_assert(I_W + 5 <= kLW && I_W + I_D - 1 + 7 <= kRWs, "staged rows too narrow for the brick");

template <bool CORR>
__global__ void __launch_bounds__(kThreads, CORR ? 2 : 4) cost_stem3d_ref3_kernel(const Ref3Params p)
{
    __shared__ float s_in[I_VOL];
    __shared__ __align__(16) float s_ab[4 * A_VOL + 4 * B_VOL];
    __shared__ float4 s_w0q[27];       // [tap] -> 4 output channels
    __shared__ float4 s_w1q[4 * 27];   // [ci][tap] -> 4 output channels
    __shared__ float s_w2[108];        // [ci][tap]
    __shared__ float s_bias[9];        // b0[4], b1[4], b2
    float* s_a = s_ab;
    float* s_b = s_ab + 4 * A_VOL;
    float* sw0q = reinterpret_cast<float*>(s_w0q);
    float* sw1q = reinterpret_cast<float*>(s_w1q);
    const float* sb0 = s_bias;
    const float* sb1 = s_bias + 4;
    const float* sb2 = s_bias + 8;
    const __half *w0 = p.w0, *b0 = p.b0, *w1 = p.w1, *b1 = p.b1, *w2 = p.w2, *b2 = p.b2;
    __half* out = p.out;
    const int D = p.D, H = p.H, W = p.W;

    const int tid = threadIdx.x;
    const int b = blockIdx.z / p.n_dtiles;
    const int od0 = (blockIdx.z - b * p.n_dtiles) * TD;
    const int oh0 = blockIdx.y * TH;
    const int ow0 = blockIdx.x * TW;
    const int64_t vol = i64(D) * H * W;

    // w0 [co][27] -> s_w0q[tap].co; w1 [co][ci][27] -> s_w1q[ci * 27 + tap].co.
    // All of a thread's global loads are issued before its first shared store.
    {
        constexpr int kIt = (kWeights + kThreads - 1) / kThreads;
        __half v[kIt];
#pragma unroll
        for (int k = 0; k < kIt; ++k) {
            const int i = tid + k * kThreads;
            const __half* src_w = i < 108 ? w0 + i : i < 112 ? b0 + (i - 108) : i < 544 ? w1 + (i - 112)
                                : i < 548 ? b1 + (i - 544) : i < 656 ? w2 + (i - 548) : b2;
            v[k] = i < kWeights ? *src_w : __float2half_rn(0.0f);
        }
#pragma unroll
        for (int k = 0; k < kIt; ++k) {
            const int i = tid + k * kThreads;
            const float f = __half2float(v[k]);
            if (i < 108) {
                const int co = i / 27, tap = i - co * 27;
                sw0q[tap * 4 + co] = f;
            } else if (i < 112) {
                s_bias[i - 108] = f;
            } else if (i < 544) {
                const int r = i - 112, co = r / 108, q = r - co * 108;  // q = ci * 27 + tap
                sw1q[q * 4 + co] = f;
            } else if (i < 548) {
                s_bias[4 + i - 544] = f;
            } else if (i < 656) {
                s_w2[i - 548] = f;
            } else if (i < kWeights) {
                s_bias[8] = f;
            }
        }
    }
    // Input brick, origin (od0-3, oh0-3, ow0-3), zero outside the volume.
    if constexpr (!CORR) {
        const __half* src = p.in + i64(b) * vol;
        constexpr int kIt = (I_VOL + kThreads - 1) / kThreads;
        __half v[kIt];
#pragma unroll
        for (int k = 0; k < kIt; ++k) {
            const int i = tid + k * kThreads;
            const int z = i / (I_H * I_W), r = i - z * I_H * I_W, y = r / I_W, x = r - y * I_W;
            const int gd = od0 - 3 + z, gh = oh0 - 3 + y, gw = ow0 - 3 + x;
            v[k] = (i < I_VOL && inside(gd, gh, gw, D, H, W)) ? src[(i64(gd) * H + gh) * W + gw]
                                                               : __float2half_rn(0.0f);
        }
#pragma unroll
        for (int k = 0; k < kIt; ++k) {
            const int i = tid + k * kThreads;
            if (i < I_VOL) s_in[i] = __half2float(v[k]);
        }
    } else {
        // The brick is the correlation volume itself, computed here with the
        // arithmetic of the bit-exact correlation kernel: per value an fp32
        // fma chain over the channels in order from +0, then acc / C or
        // acc * (1 / C) (the reference's rule for this call), fp16 rounding;
        // +0 where w - d < 0.  Thread (y, x) < (14, 14) owns the brick's 10
        // disparities at that position: one left value and 10 right values
        // (a contiguous run of the right row) per channel.
        __half* Lt = reinterpret_cast<__half*>(s_ab);  // [kCorrC][14][24]
        __half* Rt = Lt + kCorrC * I_H * kLW;          // [kCorrC][14][32]
        const int lw0 = ow0 - 8;                       // ow0 is a multiple of 8
        const int rw0 = ow0 - od0 - 9;                 // image column of w - d for (x, z) = (0, 9)
        const int rwa = rw0 & ~7;                      // floor to a multiple of 8
        const int ro = rw0 - rwa;                      // 0..7
        const int64_t plane = i64(H) * W;
        const __half* lsrc = p.left + i64(b) * p.C * plane;
        const __half* rsrc = p.right + i64(b) * p.C * plane;
        const int y = tid / I_W, x = tid - y * I_W;  // valid for tid < 196
        float acc[I_D];
#pragma unroll
        for (int z = 0; z < I_D; ++z) acc[z] = 0.0f;
        for (int c0 = 0; c0 < p.C; c0 += kCorrC) {
            const int nc = min(kCorrC, p.C - c0);
            uint4 v[kStageIt];
#pragma unroll
            for (int k = 0; k < kStageIt; ++k) {
                const int i = tid + k * kThreads;
                v[k] = make_uint4(0u, 0u, 0u, 0u);
                if (i < nc * kSegC) {
                    const int c = i / kSegC, r = i - c * kSegC;
                    const bool is_l = r < kLSeg;
                    const int rr = is_l ? r : r - kLSeg;
                    const int per_row = is_l ? kLW / 8 : kRWs / 8;
                    const int yy = rr / per_row, seg = rr - yy * per_row;
                    const int gh = oh0 - 3 + yy, gx = (is_l ? lw0 : rwa) + 8 * seg;
                    if (gh >= 0 && gh < H) {
                        const __half* src = (is_l ? lsrc : rsrc) + i64(c0 + c) * plane + i64(gh) * W;
                        if (p.vec_ok && gx >= 0 && gx + 8 <= W) {
                            v[k] = __ldg(reinterpret_cast<const uint4*>(src + gx));
                        } else {
                            __half e[8];
#pragma unroll
                            for (int q = 0; q < 8; ++q) {
                                const int g = gx + q;
                                e[q] = (g >= 0 && g < W) ? src[g] : __float2half_rn(0.0f);
                            }
                            v[k] = *reinterpret_cast<const uint4*>(e);
                        }
                    }
                }
            }
            __syncthreads();  // the previous chunk's tiles are consumed
#pragma unroll
            for (int k = 0; k < kStageIt; ++k) {
                const int i = tid + k * kThreads;
                if (i < nc * kSegC) {
                    const int c = i / kSegC, r = i - c * kSegC;
                    __half* dst = r < kLSeg ? Lt + c * (I_H * kLW) + r * 8 : Rt + c * (I_H * kRWs) + (r - kLSeg) * 8;
                    *reinterpret_cast<uint4*>(dst) = v[k];
                }
            }
            __syncthreads();
            if (tid < kLTile) {
                for (int c = 0; c < nc; ++c) {
                    const float lv = __half2float(Lt[c * (I_H * kLW) + y * kLW + x + 5]);
                    // right column of disparity z: w - d = rw0 + (x - z) + 9
                    const __half* rrow = Rt + c * (I_H * kRWs) + y * kRWs + ro + x;
#pragma unroll
                    for (int z = 0; z < I_D; ++z) acc[z] = __fmaf_rn(lv, __half2float(rrow[9 - z]), acc[z]);
                }
            }
        }
        if (tid < kLTile) {
#pragma unroll
            for (int z = 0; z < I_D; ++z) {
                const int gd = od0 - 3 + z, gh = oh0 - 3 + y, gw = ow0 - 3 + x;
                float v = 0.0f;
                if (inside(gd, gh, gw, D, H, W) && gw >= gd) {
                    const float sc = p.scale_div ? div_int(acc[z], p.C, p.inv_c) : __fmul_rn(acc[z], p.inv_c);
                    v = __half2float(__float2half_rn(sc));
                }
                s_in[(z * I_H + y) * I_W + x] = v;
            }
        }
    }
    __syncthreads();

    // Stage 0: 1 -> 4 over the stage-0 brick, origin (od0-2, oh0-2, ow0-2);
    // runs of 6 along the 12-wide rows, all 4 channels per thread (192 runs).
    {
        constexpr int NX = 6, NG = A_W / NX;
        for (int i = tid; i < A_D * A_H * NG; i += kThreads) {
            const int z = i / (A_H * NG), r = i - z * (A_H * NG), y = r / NG, x0 = (r - y * NG) * NX;
            float acc[4][NX];
            conv_run_x4<1, NX>(s_in, 0, I_H, I_W, z, y, x0, s_w0q, acc);
#pragma unroll
            for (int j = 0; j < NX; ++j) {
                const bool in_vol = inside(od0 - 2 + z, oh0 - 2 + y, ow0 - 2 + x0 + j, D, H, W);
#pragma unroll
                for (int co = 0; co < 4; ++co) {
                    const float v = __fadd_rn(acc[co][j], sb0[co]);
                    s_a[co * A_VOL + (z * A_H + y) * A_W + x0 + j] =
                        in_vol ? __half2float(__float2half_rn(relu6(v))) : 0.0f;
                }
            }
        }
    }
    __syncthreads();

    // Stage 1: 4 -> 4 over the stage-1 brick, origin (od0-1, oh0-1, ow0-1);
    // runs of 5 along the 10-wide rows, all 4 channels per thread (120 runs).
    {
        constexpr int NX = 5, NG = B_W / NX;
        for (int i = tid; i < B_D * B_H * NG; i += kThreads) {
            const int z = i / (B_H * NG), r = i - z * (B_H * NG), y = r / NG, x0 = (r - y * NG) * NX;
            float acc[4][NX];
            conv_run_x4<4, NX>(s_a, A_VOL, A_H, A_W, z, y, x0, s_w1q, acc);
#pragma unroll
            for (int j = 0; j < NX; ++j) {
                const bool in_vol = inside(od0 - 1 + z, oh0 - 1 + y, ow0 - 1 + x0 + j, D, H, W);
#pragma unroll
                for (int co = 0; co < 4; ++co) {
                    const float v = __fadd_rn(acc[co][j], sb1[co]);
                    s_b[co * B_VOL + (z * B_H + y) * B_W + x0 + j] =
                        in_vol ? __half2float(__float2half_rn(relu6(v))) : 0.0f;
                }
            }
        }
    }
    __syncthreads();

    // Stage 2: 4 -> 1, blocks of 2 rows x 2 columns per thread (64 threads).
    // For each (ci, kd) the 4 x 4 input patch is loaded once and serves the
    // 9 (kh, kw) taps of the 4 outputs; each output's chain still runs in
    // (ci, kd, kh, kw) order.
    {
        constexpr int NX = 2, NY = 2, NG = TW / NX, NYG = TH / NY;
        if (tid < TD * NYG * NG) {
            const int z = tid / (NYG * NG), r = tid - z * (NYG * NG), y0 = (r / NG) * NY, x0 = (r % NG) * NX;
            float acc[NY][NX];
#pragma unroll
            for (int a = 0; a < NY; ++a)
#pragma unroll
                for (int j = 0; j < NX; ++j) acc[a][j] = 0.0f;
#pragma unroll
            for (int ci = 0; ci < 4; ++ci)
#pragma unroll
                for (int kd = 0; kd < 3; ++kd) {
                    float patch[NY + 2][NX + 2];
#pragma unroll
                    for (int a = 0; a < NY + 2; ++a)
#pragma unroll
                        for (int t = 0; t < NX + 2; ++t)
                            patch[a][t] = s_b[ci * B_VOL + ((z + kd) * B_H + y0 + a) * B_W + x0 + t];
#pragma unroll
                    for (int kh = 0; kh < 3; ++kh)
#pragma unroll
                        for (int kw = 0; kw < 3; ++kw) {
                            const float wv = s_w2[ci * 27 + kd * 9 + kh * 3 + kw];
#pragma unroll
                            for (int a = 0; a < NY; ++a)
#pragma unroll
                                for (int j = 0; j < NX; ++j) acc[a][j] = __fmaf_rn(patch[a + kh][j + kw], wv, acc[a][j]);
                        }
                }
            const int gd = od0 + z;
#pragma unroll
            for (int a = 0; a < NY; ++a)
#pragma unroll
                for (int j = 0; j < NX; ++j) {
                    const int gh = oh0 + y0 + a, gw = ow0 + x0 + j;
                    if (gd < D && gh < H && gw < W)
                        out[i64(b) * vol + (i64(gd) * H + gh) * W + gw] =
                            __float2half_rn(relu6(__fadd_rn(acc[a][j], sb2[0])));
                }
        }
    }
}

}  // namespace

int corr_scale_div(bool is_half, int B, int C, int H, int W, int D, int sm_count) noexcept;

namespace {

int ref3_launch(bool corr, Ref3Params& p, int B, cudaStream_t stream, const char* name) noexcept
{
    if (!p.w0 || !p.b0 || !p.w1 || !p.b1 || !p.w2 || !p.b2 || !p.out) return WW_ERR_NULL_POINTER;
    if (B < 0 || p.D < 0 || p.H < 0 || p.W < 0 || p.C < 0) return WW_ERR_INVALID_SHAPE;
    // A correlation over no channels is invalid whatever the output size
    // (as in corr_volume_launch), so C is checked before the empty-output exit.
    if (corr && p.C == 0) return WW_ERR_INVALID_SHAPE;
    if (B == 0 || p.D == 0 || p.H == 0 || p.W == 0) return WW_SUCCESS;
    p.n_dtiles = (p.D + TD - 1) / TD;
    if (static_cast<long long>(B) * p.n_dtiles > 65535 || (p.H + TH - 1) / TH > 65535) return WW_ERR_UNSUPPORTED;
    DeviceInfo dev;
    if (current_device_info(&dev) != WW_SUCCESS) return WW_ERR_DEVICE;
    if (corr) {
        p.scale_div = corr_scale_div(true, B, p.C, p.H, p.W, p.D, dev.sm_count);
        p.inv_c = 1.0f / static_cast<float>(p.C);
    }
    dim3 grid((p.W + TW - 1) / TW, (p.H + TH - 1) / TH, B * p.n_dtiles);
    if (corr) cost_stem3d_ref3_kernel<true><<<grid, kThreads, 0, stream>>>(p);
    else cost_stem3d_ref3_kernel<false><<<grid, kThreads, 0, stream>>>(p);
    return launch_status(name);
}

Ref3Params ref3_params(void* out, const void* w0, const void* b0, const void* w1, const void* b1, const void* w2,
                       const void* b2, int D, int H, int W) noexcept
{
    auto h = [](const void* q) { return static_cast<const __half*>(q); };
    Ref3Params p{};
    p.out = static_cast<__half*>(out);
    p.w0 = h(w0);
    p.b0 = h(b0);
    p.w1 = h(w1);
    p.b1 = h(b1);
    p.w2 = h(w2);
    p.b2 = h(b2);
    p.D = D;
    p.H = H;
    p.W = W;
    return p;
}

}  // namespace

int cost_stem3d_ref3_launch(const void* in, void* out, const void* w0, const void* b0,
                            const void* w1, const void* b1, const void* w2, const void* b2,
                            int B, int D, int H, int W, cudaStream_t stream) noexcept
{
    if (!in) return WW_ERR_NULL_POINTER;
    Ref3Params p = ref3_params(out, w0, b0, w1, b1, w2, b2, D, H, W);
    p.in = static_cast<const __half*>(in);
    return ref3_launch(false, p, B, stream, "ww_cost_stem3d_ref3");
}

int corr_cost_stem3d_ref3_launch(const void* left, const void* right, void* out, const void* w0, const void* b0,
                                 const void* w1, const void* b1, const void* w2, const void* b2, int B, int C,
                                 int H, int W, int D, cudaStream_t stream) noexcept
{
    if (!left || !right) return WW_ERR_NULL_POINTER;
    Ref3Params p = ref3_params(out, w0, b0, w1, b1, w2, b2, D, H, W);
    p.left = static_cast<const __half*>(left);
    p.right = static_cast<const __half*>(right);
    p.C = C;
    p.vec_ok = W % 8 == 0 && reinterpret_cast<uintptr_t>(left) % 16 == 0 &&
               reinterpret_cast<uintptr_t>(right) % 16 == 0;
    return ref3_launch(true, p, B, stream, "ww_corr_cost_stem3d_ref3");
}

}  // namespace ww

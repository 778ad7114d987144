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
// segment of 128 columns for one (b, g) and a band of DT disparities:
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

#include "ww_common.cuh"

#include <type_traits>

namespace ww {
namespace {

constexpr int kTileW = 128;     // columns per CTA (32 threads x 4)
constexpr int kVecW = 4;        // columns per thread
constexpr int kDispPerThread = 8;
constexpr int kChunkC = 16;     // channels staged per pass

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
// into smem[nc][width], zero outside [0, W).
template <typename T>
__device__ __forceinline__ void stage_rows(T* __restrict__ dst, const T* __restrict__ src_row0,
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

template <typename T>
__global__ void __launch_bounds__(256) corr_volume_kernel(
    const T* __restrict__ left, const T* __restrict__ right, T* __restrict__ out,
    int C, int H, int W, int D, int G, int n_dband, int scale_div, float inv_cg, int vec_ok)
{
    constexpr int ND = kDispPerThread;
    const int DT = ND * blockDim.y;  // disparities per CTA
    const int RW = kTileW + DT;      // staged R width
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* Ls = reinterpret_cast<T*>(smem_raw);
    T* Rs = Ls + kChunkC * kTileW;

    const int w0 = blockIdx.x * kTileW;
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

    for (int c0 = 0; c0 < Cg; c0 += kChunkC) {
        const int nc = min(kChunkC, Cg - c0);
        stage_rows<T>(Ls, lrow + c0 * plane, plane, nc, w0, kTileW, W, vec_ok);
        stage_rows<T>(Rs, rrow + c0 * plane, plane, nc, w0 - d0 - DT, RW, W, vec_ok);
        __syncthreads();
        for (int c = 0; c < nc; ++c) {
            const T* lp = Ls + c * kTileW + wl;
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

    const float cg = static_cast<float>(Cg);
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
            else val = scale_div ? __fdiv_rn(acc[dd][v], cg) : __fmul_rn(acc[dd][v], inv_cg);
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

}  // namespace

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
    const float inv_cg = 1.0f / static_cast<float>(Cg);

    const int ny = min(8, (D + kDispPerThread - 1) / kDispPerThread);
    const int DT = ny * kDispPerThread;
    const int n_dband = (D + DT - 1) / DT;
    if (static_cast<long long>(H) * n_dband > 65535) return WW_ERR_UNSUPPORTED;
    dim3 block(32, ny);
    dim3 grid((W + kTileW - 1) / kTileW, H * n_dband, B * G);
    const size_t esize = is_half ? 2 : 4;
    const size_t smem = static_cast<size_t>(kChunkC) * (kTileW + kTileW + DT) * esize;
    const int vec_elems = is_half ? 8 : 4;
    const int vec_ok = (W % vec_elems == 0) && (reinterpret_cast<uintptr_t>(left) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(right) % 16 == 0);
    if (is_half) {
        corr_volume_kernel<__half><<<grid, block, smem, stream>>>(
            static_cast<const __half*>(left), static_cast<const __half*>(right), static_cast<__half*>(out),
            C, H, W, D, G, n_dband, scale_div, inv_cg, vec_ok);
    } else {
        corr_volume_kernel<float><<<grid, block, smem, stream>>>(
            static_cast<const float*>(left), static_cast<const float*>(right), static_cast<float*>(out),
            C, H, W, D, G, n_dband, scale_div, inv_cg, vec_ok);
    }
    return launch_status("ww_corr_volume");
}

}  // namespace ww

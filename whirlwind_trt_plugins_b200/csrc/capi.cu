// capi.cu -- extern "C" entry points of libww_trt_plugins.so (declared in
// include/ww_trt_plugins.h) plus the per-device state they share.
#include "ww_common.cuh"

#include <mutex>

namespace ww {

int corr_volume_launch(const void* left, const void* right, void* out, int dtype, int B, int C,
                       int H, int W, int D, int G, cudaStream_t stream) noexcept;
int cost_stem3d_ref3_launch(const void* in, void* out, const void* w0, const void* b0,
                            const void* w1, const void* b1, const void* w2, const void* b2,
                            int B, int D, int H, int W, cudaStream_t stream) noexcept;
int corr_cost_stem3d_ref3_launch(const void* left, const void* right, void* out, const void* w0, const void* b0,
                                 const void* w1, const void* b1, const void* w2, const void* b2, int B, int C,
                                 int H, int W, int D, cudaStream_t stream) noexcept;
int stem_tc_launch(const void* vol, const void* left, const void* right, const void* w,
                   const void* b, void* out, int B, int C, int G, int H, int W, int D, int Cout,
                   int act, int in_row0, int in_rows, int out_row0, int out_rows,
                   cudaStream_t stream) noexcept;
int stem_limits(bool fused, int C, int G, int D, int Cout, int smem_optin) noexcept;
int set_fused_corr_engine(int engine) noexcept;
int int_div_selftest(int b, unsigned long long* mismatches) noexcept;
int fused_corr_engine() noexcept;
int nv12_decode_launch(const void* nv12, void* out, int dtype, int B, int H_IN, int W_IN, int H_OUT,
                       int W_OUT, cudaStream_t stream) noexcept;
int disparity_regression_launch(const void* cost, void* out, int in_dtype, int out_dtype, int B, int D, int H,
                                int W, int mode, cudaStream_t stream) noexcept;

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_dev_mu;
DeviceInfo g_dev[kMaxDevices];
int* g_err_slot[kMaxDevices];

}  // namespace

// Written by bounded device-side waits that expire (see umma.cuh).
__device__ int g_ww_device_error;

int current_device_info(DeviceInfo* out) noexcept
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return WW_ERR_DEVICE;
    std::lock_guard<std::mutex> lock(g_dev_mu);
    DeviceInfo& d = g_dev[dev];
    if (d.sm_count == 0) {
        int sms = 0, smem = 0, major = 0, minor = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
            cudaGetLastError();
            return WW_ERR_DEVICE;
        }
        d.sm_count = sms;
        d.smem_optin = smem;
        d.cc_major = major;
        d.cc_minor = minor;
    }
    *out = d;
    // The kernels are built for sm_100a only, which runs on compute capability 10.0.
    return (d.cc_major == 10 && d.cc_minor == 0) ? WW_SUCCESS : WW_ERR_DEVICE;
}

int* device_error_slot() noexcept
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lock(g_dev_mu);
    if (g_err_slot[dev] == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_ww_device_error) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        g_err_slot[dev] = static_cast<int*>(p);
    }
    return g_err_slot[dev];
}

}  // namespace ww

extern "C" {

const char* ww_status_string(int status)
{
    switch (status) {
        case WW_SUCCESS: return "success";
        case WW_ERR_LAUNCH: return "CUDA launch or runtime call failed";
        case WW_ERR_INVALID_SHAPE: return "invalid tensor shape";
        case WW_ERR_INVALID_DTYPE: return "unsupported data type";
        case WW_ERR_NULL_POINTER: return "null pointer";
        case WW_ERR_UNSUPPORTED: return "request outside the supported limits";
        case WW_ERR_MISALIGNED: return "pointer not aligned as required";
        case WW_ERR_DEVICE: return "no usable sm_100 device";
        default: return "unknown status";
    }
}

int ww_abi_version(void) { return WW_ABI_VERSION; }

int ww_corr_volume(const void* left, const void* right, void* out, int dtype, int B, int C, int H,
                   int W, int D, int G, void* stream)
{
    return ww::corr_volume_launch(left, right, out, dtype, B, C, H, W, D, G,
                                  static_cast<cudaStream_t>(stream));
}

// Opt-in shared memory per block of the current device, or of a B200 when
// no usable device is current (a host checking shapes without a GPU).
static int smem_optin_or_b200() noexcept
{
    ww::DeviceInfo d;
    if (ww::current_device_info(&d) == WW_SUCCESS) return d.smem_optin;
    cudaGetLastError();
    return 232448;
}

int ww_selftest_int_division(int divisor, unsigned long long* mismatches)
{
    return ww::int_div_selftest(divisor, mismatches);
}

int ww_set_fused_corr_engine(int engine)
{
    return ww::set_fused_corr_engine(engine);
}

int ww_get_fused_corr_engine(void)
{
    return ww::fused_corr_engine();
}

int ww_corr_cost_stem3d_supported(int C, int G, int D, int Cout)
{
    return ww::stem_limits(true, C, G, D, Cout, smem_optin_or_b200());
}

int ww_cost_stem3d_supported(int Cin, int D, int Cout)
{
    return ww::stem_limits(false, Cin, Cin, D, Cout, smem_optin_or_b200());
}

int ww_cost_stem3d_ref3(const void* in, void* out, const void* w0, const void* b0, const void* w1,
                        const void* b1, const void* w2, const void* b2, int B, int D, int H, int W,
                        void* stream)
{
    return ww::cost_stem3d_ref3_launch(in, out, w0, b0, w1, b1, w2, b2, B, D, H, W,
                                       static_cast<cudaStream_t>(stream));
}

int ww_cost_stem3d(const void* vol, const void* w, const void* b, void* out, int B, int Cin, int Cout,
                   int D, int H, int W, int act, void* stream)
{
    if (vol == nullptr) return WW_ERR_NULL_POINTER;
    return ww::stem_tc_launch(vol, nullptr, nullptr, w, b, out, B, Cin, Cin, H, W, D, Cout, act, 0, H,
                              0, H, static_cast<cudaStream_t>(stream));
}

int ww_corr_cost_stem3d(const void* left, const void* right, const void* w, const void* b, void* out,
                        int B, int C, int G, int H, int W, int D, int Cout, int act, void* stream)
{
    if (left == nullptr || right == nullptr) return WW_ERR_NULL_POINTER;
    return ww::stem_tc_launch(nullptr, left, right, w, b, out, B, C, G, H, W, D, Cout, act, 0, H, 0, H,
                              static_cast<cudaStream_t>(stream));
}

int ww_corr_cost_stem3d_band(const void* left, const void* right, const void* w, const void* b,
                             void* out, int B, int C, int G, int H, int W, int D, int Cout, int act,
                             int in_row0, int in_rows, int out_row0, int out_rows, void* stream)
{
    if (left == nullptr || right == nullptr) return WW_ERR_NULL_POINTER;
    return ww::stem_tc_launch(nullptr, left, right, w, b, out, B, C, G, H, W, D, Cout, act, in_row0,
                              in_rows, out_row0, out_rows, static_cast<cudaStream_t>(stream));
}

int ww_corr_cost_stem3d_ref3(const void* left, const void* right, void* out, const void* w0, const void* b0,
                             const void* w1, const void* b1, const void* w2, const void* b2, int B, int C, int H,
                             int W, int D, void* stream)
{
    return ww::corr_cost_stem3d_ref3_launch(left, right, out, w0, b0, w1, b1, w2, b2, B, C, H, W, D,
                                            static_cast<cudaStream_t>(stream));
}

int ww_nv12_decode(const void* nv12, void* out, int dtype, int B, int H_IN, int W_IN, int H_OUT, int W_OUT,
                   void* stream)
{
    return ww::nv12_decode_launch(nv12, out, dtype, B, H_IN, W_IN, H_OUT, W_OUT,
                                  static_cast<cudaStream_t>(stream));
}

int ww_disparity_regression(const void* cost, void* out, int in_dtype, int out_dtype, int B, int D, int H, int W,
                            int mode, void* stream)
{
    return ww::disparity_regression_launch(cost, out, in_dtype, out_dtype, B, D, H, W, mode,
                                           static_cast<cudaStream_t>(stream));
}

int ww_fold_bn_f16(const float* w, const float* scale, const float* bias, int cout, int k,
                   uint16_t* w16, uint16_t* b16)
{
    if (!w || !scale || !bias || !w16 || !b16) return WW_ERR_NULL_POINTER;
    if (cout <= 0 || k <= 0) return WW_ERR_INVALID_SHAPE;
    for (int o = 0; o < cout; ++o) {
        for (int i = 0; i < k; ++i) {
            const __half h = __float2half_rn(w[static_cast<size_t>(o) * k + i] * scale[o]);
            w16[static_cast<size_t>(o) * k + i] = __half_as_ushort(h);
        }
        b16[o] = __half_as_ushort(__float2half_rn(bias[o]));
    }
    return WW_SUCCESS;
}

int ww_device_error(int* code)
{
    if (code == nullptr) return WW_ERR_NULL_POINTER;
    int* slot = ww::device_error_slot();
    if (slot == nullptr) return WW_ERR_DEVICE;
    if (cudaMemcpy(code, slot, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        return WW_ERR_LAUNCH;
    }
    return WW_SUCCESS;
}

int ww_clear_device_error(void)
{
    int* slot = ww::device_error_slot();
    if (slot == nullptr) return WW_ERR_DEVICE;
    if (cudaMemset(slot, 0, sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        return WW_ERR_LAUNCH;
    }
    return WW_SUCCESS;
}

}  // extern "C"

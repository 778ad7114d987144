// ref_capi.cu -- C entry points over the reference's own CUDA launchers.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together
// with the UNMODIFIED reference kernel sources, read in place from the
// reference tree (src/plugins/corr_volume/corr_volume_kernel.cu,
// src/plugins/cost_stem_3d/cost_stem_3d_kernel.cu and
// src/plugins/nv12_decode/nv12_decode_kernel.cu), into
// oracle/_ref/libww_ref.so.  tests/golden/make_golden.py and the GPU parity
// tests call it to pin the CPU oracle and the product against the
// reference's actual results; bench.py may time it for context.  Nothing in
// the product links it.
//
// The reference has no group-wise correlation.  wwref_corr_volume_grouped
// reproduces it with the reference kernel the only way the reference can:
// one launchCorrVolume<__half> call per (batch, group) on the contiguous
// channel slice of that group (corr_volume_kernel.hpp:17-27 takes NCHW
// pointers, and a group's channels are contiguous in NCHW).

#include "plugins/corr_volume/corr_volume_kernel.hpp"
#include "plugins/cost_stem_3d/cost_stem_3d_kernel.hpp"
#include "plugins/nv12_decode/nv12_decode_kernel.hpp"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

extern "C" {

int wwref_corr_volume_f16(const void* left, const void* right, void* out,
                          int B, int C, int H, int W, int D, void* stream)
{
    return static_cast<int>(whirlwind::launchCorrVolume<__half>(
        static_cast<const __half*>(left), static_cast<const __half*>(right),
        static_cast<__half*>(out), B, C, H, W, D, static_cast<cudaStream_t>(stream)));
}

int wwref_corr_volume_f32(const void* left, const void* right, void* out,
                          int B, int C, int H, int W, int D, void* stream)
{
    return static_cast<int>(whirlwind::launchCorrVolume<float>(
        static_cast<const float*>(left), static_cast<const float*>(right),
        static_cast<float*>(out), B, C, H, W, D, static_cast<cudaStream_t>(stream)));
}

// out[b, g, d, h, w] for G groups via B*G reference calls with B = 1.
int wwref_corr_volume_grouped_f16(const void* left, const void* right, void* out,
                                  int B, int C, int H, int W, int D, int G, void* stream)
{
    if (G <= 0 || C % G != 0) return static_cast<int>(cudaErrorInvalidValue);
    const int Cg = C / G;
    const long long plane = static_cast<long long>(H) * W;
    const __half* L = static_cast<const __half*>(left);
    const __half* R = static_cast<const __half*>(right);
    __half* O = static_cast<__half*>(out);
    for (int b = 0; b < B; ++b)
        for (int g = 0; g < G; ++g) {
            const long long in_off = (static_cast<long long>(b) * C + static_cast<long long>(g) * Cg) * plane;
            const long long out_off = (static_cast<long long>(b) * G + g) * D * plane;
            cudaError_t e = whirlwind::launchCorrVolume<__half>(
                L + in_off, R + in_off, O + out_off, 1, Cg, H, W, D, static_cast<cudaStream_t>(stream));
            if (e != cudaSuccess) return static_cast<int>(e);
        }
    return 0;
}

// NV12 decode of one image (the reference launcher takes no batch).
int wwref_nv12_decode_f16(const void* nv12, void* out, int H_IN, int W_IN, int H_OUT, int W_OUT, void* stream)
{
    return static_cast<int>(whirlwind::launchNv12Decode<__half>(static_cast<const uint8_t*>(nv12),
                                                                 static_cast<__half*>(out), H_IN, W_IN, H_OUT,
                                                                 W_OUT, static_cast<cudaStream_t>(stream)));
}

int wwref_nv12_decode_f32(const void* nv12, void* out, int H_IN, int W_IN, int H_OUT, int W_OUT, void* stream)
{
    return static_cast<int>(whirlwind::launchNv12Decode<float>(static_cast<const uint8_t*>(nv12),
                                                                static_cast<float*>(out), H_IN, W_IN, H_OUT,
                                                                W_OUT, static_cast<cudaStream_t>(stream)));
}

int wwref_cost_stem3d(const void* in, void* out,
                      const void* w0, const void* b0, const void* w1, const void* b1,
                      const void* w2, const void* b2, int B, int D, int H, int W, void* stream)
{
    auto h = [](const void* p) { return static_cast<const __half*>(p); };
    return static_cast<int>(whirlwind::launchCostStem3D(
        h(in), static_cast<__half*>(out), h(w0), h(b0), h(w1), h(b1), h(w2), h(b2),
        B, D, H, W, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"

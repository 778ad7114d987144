// plugin_core.cpp -- the logic of the reference's IPluginV3 methods for
// CorrVolume and CostStem3D (and the fused CorrCostStem3D extension), written
// against plain descriptors (ww_tensor_desc_t) instead of TensorRT types.
// The TensorRT shim in trt/ forwards each IPluginV3 method here; the tests
// call these directly.  Nothing here touches the GPU except the *_enqueue
// functions, and those only after every check has passed.
#include "../../include/ww_trt_plugins.h"

#include <cstring>

namespace {

bool is_linear_half(const ww_tensor_desc_t& d)
{
    return d.format == WW_FORMAT_LINEAR && d.dtype == WW_DTYPE_HALF;
}

bool fits_int(int64_t v) { return v >= 0 && v <= 0x7fffffff; }

bool same_shape(const ww_tensor_desc_t& a, const ww_tensor_desc_t& b)
{
    if (a.nb_dims != b.nb_dims || a.nb_dims < 0 || a.nb_dims > 8) return false;
    for (int i = 0; i < a.nb_dims; ++i)
        if (a.dims[i] != b.dims[i]) return false;
    return true;
}

// Element count of a descriptor; -1 for a negative (unknown) or invalid shape.
int64_t numel(const ww_tensor_desc_t& d)
{
    if (d.nb_dims < 0 || d.nb_dims > 8) return -1;
    int64_t n = 1;
    for (int i = 0; i < d.nb_dims; ++i) {
        if (d.dims[i] < 0) return -1;
        n *= d.dims[i];
    }
    return n;
}

}  // namespace

extern "C" {

// plugin_fields.hpp:17-31: first field named `name` whose data is non-null.
int ww_plugin_get_int_field(int nb_fields, const char* const* names, const int32_t* const* values,
                            const char* name, int fallback)
{
    if (names == nullptr || values == nullptr || name == nullptr) return fallback;
    for (int i = 0; i < nb_fields; ++i) {
        if (values[i] == nullptr || names[i] == nullptr) continue;
        if (std::strcmp(names[i], name) == 0) return *values[i];
    }
    return fallback;
}

// ---------------------------------------------------------------- CorrVolume

// corr_volume.cpp:28-37: output type = input 0 type.
int ww_plugin_corr_volume_output_dtype(int nb_inputs, const int32_t* in_dtypes, int32_t* out_dtype)
{
    if (nb_inputs < 1 || in_dtypes == nullptr || out_dtype == nullptr) return 1;
    *out_dtype = in_dtypes[0];
    return 0;
}

// corr_volume.cpp:39-58: [B, max_disp, H, W]; with the num_groups extension
// and G > 1: [B, G, max_disp, H, W].
int ww_plugin_corr_volume_output_dims(int max_disp, int num_groups, int nb_inputs,
                                      const ww_tensor_desc_t* inputs, ww_tensor_desc_t* out)
{
    if (nb_inputs != 2 || inputs == nullptr || out == nullptr) return 1;
    const ww_tensor_desc_t& in = inputs[0];
    if (in.nb_dims != 4) return 1;
    *out = in;
    if (num_groups <= 1) {
        out->nb_dims = 4;
        out->dims[0] = in.dims[0];
        out->dims[1] = max_disp;
        out->dims[2] = in.dims[2];
        out->dims[3] = in.dims[3];
    } else {
        out->nb_dims = 5;
        out->dims[0] = in.dims[0];
        out->dims[1] = num_groups;
        out->dims[2] = max_disp;
        out->dims[3] = in.dims[2];
        out->dims[4] = in.dims[3];
    }
    return 0;
}

// corr_volume.cpp:60-82: LINEAR only; position 0 fp16 only (advertising
// fp32 would let TensorRT insert a reformat in front of the fast path); the
// other input and the output must match position 0.
int ww_plugin_corr_volume_supports_format(int pos, const ww_tensor_desc_t* in_out, int nb_inputs,
                                          int nb_outputs)
{
    if (in_out == nullptr || nb_inputs != 2 || nb_outputs != 1) return 0;
    if (pos < 0 || pos >= nb_inputs + nb_outputs) return 0;
    const ww_tensor_desc_t& d = in_out[pos];
    if (d.format != WW_FORMAT_LINEAR) return 0;
    if (pos == 0) return d.dtype == WW_DTYPE_HALF;
    return d.dtype == in_out[0].dtype;
}

// corr_volume.cpp:84-111: rank-4 input, fp16 or fp32, launch; 0 or 1.
int ww_plugin_corr_volume_enqueue(int max_disp, int num_groups, const ww_tensor_desc_t* in_desc,
                                  const void* const* inputs, void* const* outputs, void* stream)
{
    if (in_desc == nullptr || inputs == nullptr || outputs == nullptr) return 1;
    const ww_tensor_desc_t& d = in_desc[0];
    if (d.nb_dims != 4) return 1;
    for (int i = 0; i < 4; ++i)
        if (!fits_int(d.dims[i])) return 1;
    if (d.dtype != WW_DTYPE_HALF && d.dtype != WW_DTYPE_FLOAT) return 1;
    const int G = num_groups <= 0 ? 1 : num_groups;
    const int st = ww_corr_volume(inputs[0], inputs[1], outputs[0], d.dtype, static_cast<int>(d.dims[0]),
                                  static_cast<int>(d.dims[1]), static_cast<int>(d.dims[2]),
                                  static_cast<int>(d.dims[3]), max_disp, G, stream);
    return st == WW_SUCCESS ? 0 : 1;
}

// ---------------------------------------------------------------- CostStem3D

// cost_stem_3d.cpp:28-37 (7 inputs: output = input 0 shape) plus the 3-input
// generalised form (output [B, Cout, D, H, W], Cout = w.dims[0]).
int ww_plugin_cost_stem3d_output_dims(int nb_inputs, const ww_tensor_desc_t* inputs, ww_tensor_desc_t* out)
{
    if (inputs == nullptr || out == nullptr) return 1;
    if (nb_inputs == 7) {
        *out = inputs[0];
        return 0;
    }
    if (nb_inputs == 3) {
        if (inputs[0].nb_dims != 5 || inputs[1].nb_dims != 5) return 1;
        // the generalised stem's limits (ww_cost_stem3d_supported), where known
        const int64_t Cin = inputs[0].dims[1], D = inputs[0].dims[2], Cout = inputs[1].dims[0];
        if (Cin > 0 && D > 0 && Cout > 0 && fits_int(Cin) && fits_int(D) && fits_int(Cout) &&
            ww_cost_stem3d_supported(static_cast<int>(Cin), static_cast<int>(D), static_cast<int>(Cout)) != WW_SUCCESS)
            return 1;
        *out = inputs[0];
        out->dims[1] = inputs[1].dims[0];
        return 0;
    }
    return 1;
}

// cost_stem_3d.cpp:39-48: every position fp16 LINEAR.
int ww_plugin_cost_stem3d_supports_format(int pos, const ww_tensor_desc_t* in_out, int nb_inputs,
                                          int nb_outputs)
{
    if (in_out == nullptr || (nb_inputs != 7 && nb_inputs != 3) || nb_outputs != 1) return 0;
    if (pos < 0 || pos >= nb_inputs + nb_outputs) return 0;
    return is_linear_half(in_out[pos]);
}

// cost_stem_3d.cpp:50-73 (rank-5 input 0, B = d[0], D = d[2], H = d[3],
// W = d[4]) and the 3-input form (w [Cout, Cin, 3, 3, 3], b [Cout]).
int ww_plugin_cost_stem3d_enqueue(int nb_inputs, int act, const ww_tensor_desc_t* in_desc,
                                  const void* const* inputs, void* const* outputs, void* stream)
{
    if (in_desc == nullptr || inputs == nullptr || outputs == nullptr) return 1;
    const ww_tensor_desc_t& d = in_desc[0];
    if (d.nb_dims != 5) return 1;
    for (int i = 0; i < 5; ++i)
        if (!fits_int(d.dims[i])) return 1;
    const int B = static_cast<int>(d.dims[0]), D = static_cast<int>(d.dims[2]);
    const int H = static_cast<int>(d.dims[3]), W = static_cast<int>(d.dims[4]);
    int st;
    if (nb_inputs == 7) {
        st = ww_cost_stem3d_ref3(inputs[0], outputs[0], inputs[1], inputs[2], inputs[3], inputs[4], inputs[5],
                                 inputs[6], B, D, H, W, stream);
    } else if (nb_inputs == 3) {
        const ww_tensor_desc_t& wd = in_desc[1];
        if (wd.nb_dims != 5 || wd.dims[1] != d.dims[1] || wd.dims[2] != 3 || wd.dims[3] != 3 || wd.dims[4] != 3)
            return 1;
        if (!fits_int(wd.dims[0])) return 1;
        st = ww_cost_stem3d(inputs[0], inputs[1], inputs[2], outputs[0], B, static_cast<int>(d.dims[1]),
                            static_cast<int>(wd.dims[0]), D, H, W, act, stream);
    } else {
        return 1;
    }
    return st == WW_SUCCESS ? 0 : 1;
}

// ------------------------------------------------------- CorrCostStem3D (new)

int ww_plugin_corr_cost_stem3d_output_dims(int max_disp, int num_groups, int nb_inputs,
                                           const ww_tensor_desc_t* inputs, ww_tensor_desc_t* out)
{
    if ((nb_inputs != 4 && nb_inputs != 8) || inputs == nullptr || out == nullptr) return 1;
    if (inputs[0].nb_dims != 4) return 1;
    if (nb_inputs == 4) {
        // The fused kernel's limits, checked here so that an engine build
        // fails rather than the enqueue (C may be unknown, -1, for a dynamic
        // shape: then the group-size dependent part is left to the enqueue).
        if (inputs[2].nb_dims != 5) return 1;
        const int G = num_groups <= 0 ? 1 : num_groups;
        if (inputs[2].dims[1] != G || !fits_int(inputs[2].dims[0])) return 1;
        const int Cout = static_cast<int>(inputs[2].dims[0]);
        const int64_t C = inputs[0].dims[1];
        const int lim = C > 0 && fits_int(C) ? ww_corr_cost_stem3d_supported(static_cast<int>(C), G, max_disp, Cout)
                                             : ww_corr_cost_stem3d_supported(8 * G, G, max_disp, Cout);
        if (lim != WW_SUCCESS) return 1;
    }
    *out = inputs[0];
    out->nb_dims = 5;
    out->dims[0] = inputs[0].dims[0];
    // 8 inputs: the reference's 3-stage stem (w0, b0, w1, b1, w2, b2), one
    // output channel
    out->dims[1] = nb_inputs == 8 ? 1 : inputs[2].dims[0];
    out->dims[2] = max_disp;
    out->dims[3] = inputs[0].dims[2];
    out->dims[4] = inputs[0].dims[3];
    return 0;
}

int ww_plugin_corr_cost_stem3d_supports_format(int pos, const ww_tensor_desc_t* in_out, int nb_inputs,
                                               int nb_outputs)
{
    if (in_out == nullptr || (nb_inputs != 4 && nb_inputs != 8) || nb_outputs != 1) return 0;
    if (pos < 0 || pos >= nb_inputs + nb_outputs) return 0;
    return is_linear_half(in_out[pos]);
}

int ww_plugin_corr_cost_stem3d_enqueue(int nb_inputs, int max_disp, int num_groups, int act,
                                       const ww_tensor_desc_t* in_desc, const void* const* inputs,
                                       void* const* outputs, void* stream)
{
    if (in_desc == nullptr || inputs == nullptr || outputs == nullptr) return 1;
    if (nb_inputs != 4 && nb_inputs != 8) return 1;
    const ww_tensor_desc_t& d = in_desc[0];
    if (d.nb_dims != 4 || !same_shape(d, in_desc[1])) return 1;
    for (int i = 0; i < 4; ++i)
        if (!fits_int(d.dims[i])) return 1;
    for (int i = 0; i < nb_inputs; ++i)
        if (in_desc[i].dtype != WW_DTYPE_HALF) return 1;
    if (nb_inputs == 8) {
        // CorrVolume (G = 1) fused with the reference's 3-stage CostStem3D:
        // w0 [4,1,3,3,3] b0 [4] w1 [4,4,3,3,3] b1 [4] w2 [1,4,3,3,3] b2 [1]
        // (cost_stem_3d_kernel.hpp:8-15), any rank with those element
        // counts; num_groups must be 1 and the activation is ReLU6.
        static const int64_t kCounts[6] = {108, 4, 432, 4, 108, 1};
        if (num_groups > 1) return 1;
        for (int i = 0; i < 6; ++i)
            if (numel(in_desc[2 + i]) != kCounts[i]) return 1;
        const int st = ww_corr_cost_stem3d_ref3(inputs[0], inputs[1], outputs[0], inputs[2], inputs[3], inputs[4],
                                                inputs[5], inputs[6], inputs[7], static_cast<int>(d.dims[0]),
                                                static_cast<int>(d.dims[1]), static_cast<int>(d.dims[2]),
                                                static_cast<int>(d.dims[3]), max_disp, stream);
        return st == WW_SUCCESS ? 0 : 1;
    }
    const ww_tensor_desc_t& wd = in_desc[2];
    const int G = num_groups <= 0 ? 1 : num_groups;
    if (wd.nb_dims != 5 || wd.dims[1] != G || wd.dims[2] != 3 || wd.dims[3] != 3 || wd.dims[4] != 3 ||
        !fits_int(wd.dims[0]))
        return 1;
    if (numel(in_desc[3]) != wd.dims[0]) return 1;  // one bias per output channel
    const int st = ww_corr_cost_stem3d(inputs[0], inputs[1], inputs[2], inputs[3], outputs[0],
                                       static_cast<int>(d.dims[0]), static_cast<int>(d.dims[1]), G,
                                       static_cast<int>(d.dims[2]), static_cast<int>(d.dims[3]), max_disp,
                                       static_cast<int>(wd.dims[0]), act, stream);
    return st == WW_SUCCESS ? 0 : 1;
}

// ------------------------------------------------------------- Nv12Decode

// nv12_decode.cpp:26-39: the output is declared fp32 whatever the input
// (TensorRT picks fp16 or fp32 through supportsFormatCombination).
int ww_plugin_nv12_decode_output_dtype(int nb_inputs, int32_t* out_dtype)
{
    (void)nb_inputs;
    if (out_dtype == nullptr) return 1;
    *out_dtype = WW_DTYPE_FLOAT;
    return 0;
}

// nv12_decode.cpp:41-60: [B, H_IN * 3 / 2, W_IN] -> [B, 3, out_h, out_w].
int ww_plugin_nv12_decode_output_dims(int out_h, int out_w, int nb_inputs, const ww_tensor_desc_t* inputs,
                                      ww_tensor_desc_t* out)
{
    if (nb_inputs != 1 || inputs == nullptr || out == nullptr) return 1;
    *out = inputs[0];
    out->nb_dims = 4;
    out->dims[0] = inputs[0].dims[0];
    out->dims[1] = 3;
    out->dims[2] = out_h;
    out->dims[3] = out_w;
    out->dtype = WW_DTYPE_FLOAT;
    return 0;
}

// nv12_decode.cpp:62-86: LINEAR; position 0 INT8 only (the bytes are uint8
// NV12 values; accepting fp32 would let TensorRT insert a sign-extending
// cast), the output fp16 or fp32.
int ww_plugin_nv12_decode_supports_format(int pos, const ww_tensor_desc_t* in_out, int nb_inputs, int nb_outputs)
{
    if (in_out == nullptr || nb_inputs != 1 || nb_outputs != 1) return 0;
    if (pos < 0 || pos >= nb_inputs + nb_outputs) return 0;
    const ww_tensor_desc_t& d = in_out[pos];
    if (d.format != WW_FORMAT_LINEAR) return 0;
    if (pos == 0) return d.dtype == WW_DTYPE_INT8;
    return d.dtype == WW_DTYPE_HALF || d.dtype == WW_DTYPE_FLOAT;
}

// nv12_decode.cpp:88-115: rank-3 input, H_IN = 2 d[1] / 3, W_IN = d[2]; the
// output dtype selects the kernel; 0 or 1.  Every batch item is decoded (the
// reference launches batch 0 only).
int ww_plugin_nv12_decode_enqueue(int out_h, int out_w, const ww_tensor_desc_t* in_desc,
                                  const ww_tensor_desc_t* out_desc, const void* const* inputs,
                                  void* const* outputs, void* stream)
{
    if (in_desc == nullptr || out_desc == nullptr || inputs == nullptr || outputs == nullptr) return 1;
    const ww_tensor_desc_t& d = in_desc[0];
    if (d.nb_dims != 3) return 1;
    for (int i = 0; i < 3; ++i)
        if (!fits_int(d.dims[i])) return 1;
    const int dt = out_desc[0].dtype;
    if (dt != WW_DTYPE_HALF && dt != WW_DTYPE_FLOAT) return 1;
    const int H_IN = static_cast<int>(d.dims[1] * 2 / 3);
    const int st = ww_nv12_decode(inputs[0], outputs[0], dt, static_cast<int>(d.dims[0]), H_IN,
                                  static_cast<int>(d.dims[2]), out_h, out_w, stream);
    return st == WW_SUCCESS ? 0 : 1;
}

// ------------------------------------------------------ DisparityRegression
// No reference counterpart (the reference pipeline ends at CostStem3D); the
// plugin follows the conventions of the ones above: LINEAR, output dtype =
// input dtype, 0 / 1 enqueue codes.

// [B, D, H, W] or [B, 1, D, H, W] -> [B, 1, H, W].
int ww_plugin_disparity_regression_output_dims(int nb_inputs, const ww_tensor_desc_t* inputs,
                                               ww_tensor_desc_t* out)
{
    if (nb_inputs != 1 || inputs == nullptr || out == nullptr) return 1;
    const ww_tensor_desc_t& d = inputs[0];
    if (d.nb_dims != 4 && !(d.nb_dims == 5 && d.dims[1] == 1)) return 1;
    *out = d;
    out->nb_dims = 4;
    out->dims[0] = d.dims[0];
    out->dims[1] = 1;
    out->dims[2] = d.dims[d.nb_dims - 2];
    out->dims[3] = d.dims[d.nb_dims - 1];
    return 0;
}

// Position 0 fp16 or fp32 LINEAR; the output matches the input's dtype.
int ww_plugin_disparity_regression_supports_format(int pos, const ww_tensor_desc_t* in_out, int nb_inputs,
                                                   int nb_outputs)
{
    if (in_out == nullptr || nb_inputs != 1 || nb_outputs != 1) return 0;
    if (pos < 0 || pos >= nb_inputs + nb_outputs) return 0;
    const ww_tensor_desc_t& d = in_out[pos];
    if (d.format != WW_FORMAT_LINEAR) return 0;
    if (d.dtype != WW_DTYPE_HALF && d.dtype != WW_DTYPE_FLOAT) return 0;
    return pos == 0 || d.dtype == in_out[0].dtype;
}

int ww_plugin_disparity_regression_enqueue(int mode, const ww_tensor_desc_t* in_desc,
                                           const ww_tensor_desc_t* out_desc, const void* const* inputs,
                                           void* const* outputs, void* stream)
{
    if (in_desc == nullptr || out_desc == nullptr || inputs == nullptr || outputs == nullptr) return 1;
    const ww_tensor_desc_t& d = in_desc[0];
    if (d.nb_dims != 4 && !(d.nb_dims == 5 && d.dims[1] == 1)) return 1;
    for (int i = 0; i < d.nb_dims; ++i)
        if (!fits_int(d.dims[i])) return 1;
    const int n = d.nb_dims;
    const int st = ww_disparity_regression(inputs[0], outputs[0], d.dtype, out_desc[0].dtype,
                                           static_cast<int>(d.dims[0]), static_cast<int>(d.dims[n - 3]),
                                           static_cast<int>(d.dims[n - 2]), static_cast<int>(d.dims[n - 1]), mode,
                                           stream);
    return st == WW_SUCCESS ? 0 : 1;
}

}  // extern "C"

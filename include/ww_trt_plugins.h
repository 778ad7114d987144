/*
 * ww_trt_plugins.h -- C ABI of the B200-native stereo cost-volume front end.
 *
 * One shared library, whirlwind_trt_plugins_b200/libww_trt_plugins.so, built
 * for sm_100a.  Every entry point is `extern "C"`, takes plain pointers and
 * sizes, never throws, never synchronises the device and never allocates
 * device memory; kernels are enqueued on `stream` (a cudaStream_t passed as
 * void*, NULL = legacy default stream).  Device pointers are CUDA device
 * memory of the current device.
 *
 * Reference interfaces replaced (paths relative to the reference project,
 * IntelligentRoboticsLab/whirlwind_trt_plugins):
 *   ww_corr_volume            whirlwind::launchCorrVolume<T>
 *                             src/plugins/corr_volume/corr_volume_kernel.hpp:17-27
 *   ww_cost_stem3d_ref3       whirlwind::launchCostStem3D
 *                             src/plugins/cost_stem_3d/cost_stem_3d_kernel.hpp:17-30
 *   ww_nv12_decode            whirlwind::launchNv12Decode<T>
 *                             src/plugins/nv12_decode/nv12_decode_kernel.hpp:20-28
 *   ww_plugin_*               the IPluginV3 methods of CorrVolumePlugin
 *                             (src/plugins/corr_volume/corr_volume.cpp:28-139) and
 *                             CostStem3DPlugin (src/plugins/cost_stem_3d/cost_stem_3d.cpp:19-97),
 *                             Nv12DecodePlugin (src/plugins/nv12_decode/nv12_decode.cpp:26-146),
 *                             with TensorRT types replaced by ww_tensor_desc_t
 * Extensions with no reference symbol (group-wise correlation fused with a
 * single G -> Cout 3-D conv stem):
 *   ww_cost_stem3d            generalised 3-input CostStem3D (Cin -> Cout)
 *   ww_corr_cost_stem3d       fused CorrVolume -> CostStem3D ("CorrCostStem3D")
 *   ww_corr_cost_stem3d_band  the same over a band of image rows (multi-GPU sharding)
 *
 * Status codes: 0 on success.  The plugin-level ww_plugin_*_enqueue calls
 * return exactly what IPluginV3OneRuntime::enqueue returns in the reference
 * (0 success, 1 failure; corr_volume.cpp:84-111).  The kernel-level calls
 * return a ww_status_t; on a CUDA launch failure they print
 * "[ww_trt_plugins] <function>: CUDA launch failed: <reason>" to stderr, as
 * the reference's lastLaunchError does (src/common/cuda_check.hpp:15-23).
 */
#ifndef WW_TRT_PLUGINS_H
#define WW_TRT_PLUGINS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WW_ABI_VERSION 2

typedef enum ww_status {
    WW_SUCCESS = 0,
    WW_ERR_LAUNCH = 1,        /* a CUDA launch or runtime call failed            */
    WW_ERR_INVALID_SHAPE = 2, /* a size is negative, zero where it may not be, or inconsistent */
    WW_ERR_INVALID_DTYPE = 3, /* dtype not accepted by this entry point          */
    WW_ERR_NULL_POINTER = 4,  /* a required pointer is NULL                      */
    WW_ERR_UNSUPPORTED = 5,   /* valid request outside this build's limits       */
    WW_ERR_MISALIGNED = 6,    /* a pointer lacks the alignment the kernel needs  */
    WW_ERR_DEVICE = 7         /* no usable sm_100 device is current              */
} ww_status_t;

/* Same numeric values as nvinfer1::DataType::kFLOAT / kHALF / kINT8. */
typedef enum ww_dtype { WW_DTYPE_FLOAT = 0, WW_DTYPE_HALF = 1, WW_DTYPE_INT8 = 2 } ww_dtype_t;

/* Activation of the generalised / fused stem. */
typedef enum ww_act { WW_ACT_RELU = 0, WW_ACT_RELU6 = 1 } ww_act_t;

/* Disparity regression: softmax over the disparities of +cost (similarity)
 * or -cost (matching cost). */
typedef enum ww_disp_mode { WW_DISP_SOFTARGMAX = 0, WW_DISP_SOFTARGMIN = 1 } ww_disp_mode_t;

/* Tensor format, same value as nvinfer1::TensorFormat::kLINEAR. */
#define WW_FORMAT_LINEAR 0

const char* ww_status_string(int status);
int ww_abi_version(void);

/* ---------------------------------------------------------------------------
 * CorrVolume
 *   out[b, g, d, h, w] = mean_{c in group g} left[b, c, h, w] * right[b, c, h, w - d]
 *   = +0 where w - d < 0.
 * left, right : [B, C, H, W]   dtype WW_DTYPE_HALF or WW_DTYPE_FLOAT
 * out         : [B, G, D, H, W] same dtype (G == 1 is the reference [B, D, H, W])
 * G divides C.  fp32 sum over the group's channels in channel order; the mean
 * is taken exactly as the reference kernel the call would run takes it
 * (acc / C or acc * (1/C)), so results are bit-identical to the reference
 * called once per (b, g).
 * Replaces whirlwind::launchCorrVolume<T> (corr_volume_kernel.hpp:17-27).
 * ------------------------------------------------------------------------- */
int ww_corr_volume(const void* left, const void* right, void* out, int dtype,
                   int B, int C, int H, int W, int D, int G, void* stream);

/* ---------------------------------------------------------------------------
 * CostStem3D, reference 7-input form: three Conv3d 3x3x3 pad 1 (1->4->4->1),
 * folded-BN bias, ReLU6, fp16 intermediates.  All fp16.
 * in, out : [B, 1, D, H, W];  w0 [4,1,3,3,3] b0 [4] w1 [4,4,3,3,3] b1 [4]
 * w2 [1,4,3,3,3] b2 [1].  Every batch item is computed (the reference kernel
 * writes batch 0 only, cost_stem_3d_kernel.cu:92).
 * Replaces whirlwind::launchCostStem3D (cost_stem_3d_kernel.hpp:17-30).
 * ------------------------------------------------------------------------- */
int ww_cost_stem3d_ref3(const void* in, void* out,
                        const void* w0, const void* b0, const void* w1, const void* b1,
                        const void* w2, const void* b2,
                        int B, int D, int H, int W, void* stream);

/* ---------------------------------------------------------------------------
 * Generalised CostStem3D (extension, 3-input form): one Conv3d 3x3x3 pad 1,
 * Cin -> Cout, + bias, ReLU or ReLU6.  All fp16, fp32 accumulation on the
 * tensor cores.
 * vol [B, Cin, D, H, W], w [Cout, Cin, 3, 3, 3] (BN already folded, see
 * ww_fold_bn_f16), b [Cout], out [B, Cout, D, H, W].
 * Fastest with W % 8 == 0 and a 16-byte aligned vol (staged by TMA); any
 * other volume is gathered element by element, with the same output.
 * ------------------------------------------------------------------------- */
int ww_cost_stem3d(const void* vol, const void* w, const void* b, void* out,
                   int B, int Cin, int Cout, int D, int H, int W, int act, void* stream);

/* ---------------------------------------------------------------------------
 * Fused CorrVolume -> CostStem3D (extension, "CorrCostStem3D"):
 *   vol = group-wise correlation of left and right (G groups, D disparities)
 *   out = ww_cost_stem3d(vol, w, b, act)                          [B, Cout, D, H, W]
 * left, right [B, C, H, W] fp16; w [Cout, G, 3, 3, 3] fp16; b [Cout] fp16.
 * The volume stays in shared memory (fp16, never written to device memory).
 * With the default engine it is accumulated on the tensor cores in fp32 and
 * scaled by 1/(C/G), so it may differ from ww_corr_volume's in the last fp32
 * bits (and, after fp16 rounding, by one fp16 ulp on rare values); the
 * output agrees with ww_corr_volume followed by ww_cost_stem3d to within
 * 2e-2 absolute.
 * ------------------------------------------------------------------------- */
int ww_corr_cost_stem3d(const void* left, const void* right, const void* w, const void* b,
                        void* out, int B, int C, int G, int H, int W, int D, int Cout,
                        int act, void* stream);

/* Correlation engine of the fused op (ww_corr_cost_stem3d, _band, _multi),
 * process-wide; returns the previous engine, or WW_ERR_INVALID_SHAPE for an
 * unknown value.  Takes effect for launches made after the call.
 *   WW_CORR_ENGINE_TENSOR      (default) warp-level tensor cores (mma.sync):
 *                              fp32 accumulation in the tensor core's order.
 *   WW_CORR_ENGINE_CUDA_CORES  fp32 fma of the fp16 products in channel
 *                              order: the volume equals ww_corr_volume's bit
 *                              for bit before the stem.  Measured 1.3x
 *                              (config 2) to 1.4x (config 4) slower than the
 *                              tensor engine on a B200. */
#define WW_CORR_ENGINE_TENSOR 0
#define WW_CORR_ENGINE_CUDA_CORES 1
int ww_set_fused_corr_engine(int engine);
int ww_get_fused_corr_engine(void);

/* Limits of ww_corr_cost_stem3d / _band / _multi and of ww_cost_stem3d
 * (this build): Cout <= 32; G (or Cin) <= 56 (at most 32 K-steps of two
 * 8-group chunks); and the weights, two volume rows and two staging slots
 * of a 16-disparity band within the device's shared memory, which bounds
 * wide groups (on a B200 every G <= 56 fits with C / G = 8; G = 56 with
 * C / G = 32 and Cout 17..32 does not).  Any D: a disparity range one
 * launch cannot hold (three
 * Cout-column tensor-memory accumulators per 16 disparities within 512
 * columns, i.e. more than 80 disparities for Cout 17..32 or 160 for
 * Cout <= 16, or a shared-memory layout that does not fit) runs as several
 * launches over disparity bands, each with the volume plane below and above
 * it, with the same result.  Shapes outside the limits return
 * WW_ERR_UNSUPPORTED.  These two functions answer without launching
 * anything (0, WW_ERR_INVALID_SHAPE or WW_ERR_UNSUPPORTED), using the current
 * device's shared memory, or a B200's when no usable device is current. */
int ww_corr_cost_stem3d_supported(int C, int G, int D, int Cout);
int ww_cost_stem3d_supported(int Cin, int D, int Cout);

/* Row-band form of ww_corr_cost_stem3d for sharding one image pair across
 * devices.  `left`/`right` hold image rows [in_row0, in_row0 + in_rows) of an
 * H-row image ([B, C, in_rows, W]); `out` receives rows
 * [out_row0, out_row0 + out_rows) ([B, Cout, D, out_rows, W]).  The input
 * band must cover [out_row0 - 1, out_row0 + out_rows + 1) clipped to [0, H)
 * (a one-row halo each side).  Rows outside [0, H) are the conv's zero
 * padding, exactly as in the unsharded call. */
int ww_corr_cost_stem3d_band(const void* left, const void* right, const void* w, const void* b,
                             void* out, int B, int C, int G, int H, int W, int D, int Cout,
                             int act, int in_row0, int in_rows, int out_row0, int out_rows,
                             void* stream);

/* ---------------------------------------------------------------------------
 * Multi-device driver of ww_corr_cost_stem3d (extension; the reference has no
 * multi-GPU code).  One host thread, n parts,
 * part k on device devices[k] with stream streams[k] (streams NULL: the
 * legacy default stream of each device).  Several parts may use the same
 * device.  Asynchronous: returns once everything is enqueued.
 *   WW_MULTI_BATCH  part k holds batch items [b0, b1) = split_even(B, n, k)
 *                   (the first B % n parts get one more): left[k], right[k]
 *                   [b1 - b0, C, H, W] -> out[k] [b1 - b0, Cout, D, H, W];
 *                   nothing moves between devices.
 *   WW_MULTI_ROWS   one image split by rows: part k owns rows [r0, r1) and
 *                   holds them in a band buffer left[k], right[k]
 *                   [B, C, i1 - i0, W] of rows [i0, i1) (ww_multi_split: one
 *                   halo row each side, clipped).  The caller fills the own
 *                   rows; the driver copies each halo row from the
 *                   neighbour's band (one strided cudaMemcpy3DPeerAsync per
 *                   row and tensor, on streams[k], after everything already
 *                   enqueued on the neighbour's stream), then runs the band
 *                   form: out[k] [B, Cout, D, r1 - r0, W].  Work enqueued
 *                   afterwards on a part's stream waits for the neighbours'
 *                   copies out of its rows.  The stitched rows equal
 *                   ww_corr_cost_stem3d on the whole image bit for bit.
 * w[k] [Cout, G, 3, 3, 3] and b[k] [Cout]: the weights, on device k.
 * Returns 0 or the first failing status (a failed copy: WW_ERR_LAUNCH with
 * the CUDA message on stderr); work enqueued before a failure stays enqueued.
 * ------------------------------------------------------------------------- */
#define WW_MULTI_BATCH 0
#define WW_MULTI_ROWS 1
int ww_corr_cost_stem3d_multi(int n, const int* devices, int mode, void* const* left, void* const* right,
                              const void* const* w, const void* const* b, void* const* out, int B, int C, int G,
                              int H, int W, int D, int Cout, int act, void* const* streams);

/* Row partition of the multi-device driver (host only): part k of n owns
 * image rows [r0, r1) of H (the first H % n parts get one more) and needs
 * the band [i0, i1) = [max(r0 - 1, 0), min(r1 + 1, H)).  Needs H >= n. */
int ww_multi_split(int n, int H, int k, int* r0, int* r1, int* i0, int* i1);

/* Fault injection for tests (host side): after `after_n_copies` more halo
 * copies, the next one the driver would issue fails with
 * cudaErrorInvalidValue instead of being enqueued (once); negative
 * disables.  The process-wide setting also affects concurrent callers. */
int ww_multi_inject_copy_failure(int after_n_copies);

/* Test hook: the naive CorrVolume rule divides every output by the group
 * width (corr_volume_kernel.cu:84), computed here with one correction fma
 * after a multiply by the rounded reciprocal (Markstein); this counts the
 * fp32 values a, over all 2^32 bit patterns, for which that quotient differs
 * from the IEEE rounded a / divisor (1 <= divisor <= 1024; synchronises). */
int ww_selftest_int_division(int divisor, unsigned long long* mismatches);

/* ---------------------------------------------------------------------------
 * CorrVolume (G = 1) fused with the reference's 3-stage CostStem3D, the pair
 * the reference runs at its native shape ([1, 1, 48, 32, 40]):
 *   out = ww_cost_stem3d_ref3(ww_corr_volume(left, right, D), w0 .. b2)
 * bit for bit (the correlation is computed inside the stem's bricks with the
 * same arithmetic and scale rule; the volume never reaches device memory).
 * left, right : [B, C, H, W] fp16; weights as ww_cost_stem3d_ref3;
 * out         : [B, 1, D, H, W] fp16.
 * ------------------------------------------------------------------------- */
int ww_corr_cost_stem3d_ref3(const void* left, const void* right, void* out, const void* w0, const void* b0,
                             const void* w1, const void* b1, const void* w2, const void* b2, int B, int C, int H,
                             int W, int D, void* stream);

/* ---------------------------------------------------------------------------
 * Nv12Decode: NV12 -> planar RGB in [-1, 1], bilinear resize.
 * nv12 : [B, H_IN * 3 / 2, W_IN] uint8 (Y plane, then interleaved U/V rows
 *        at half resolution); out : [B, 3, H_OUT, W_OUT], dtype
 *        WW_DTYPE_HALF or WW_DTYPE_FLOAT.  align_corners = False sampling
 *        with clamped taps, full-range BT.601 fused with 2 * (rgb / 255) - 1,
 *        fp32 arithmetic identical to the reference kernel's.  Every batch
 *        item is decoded (the reference launcher takes one image).
 * Replaces whirlwind::launchNv12Decode<T> (nv12_decode_kernel.hpp:20-28).
 * ------------------------------------------------------------------------- */
int ww_nv12_decode(const void* nv12, void* out, int dtype, int B, int H_IN, int W_IN, int H_OUT, int W_OUT,
                   void* stream);

/* ---------------------------------------------------------------------------
 * Disparity regression (soft-argmax / soft-argmin), the step after the 3-D
 * aggregation of a stereo network.  The reference library has no such op;
 * the formula below is its specification:
 *   disp[b, 0, h, w] = sum_d d * softmax_d(s * cost[b, d, h, w]),
 *   s = +1 (WW_DISP_SOFTARGMAX) or -1 (WW_DISP_SOFTARGMIN).
 * cost : [B, D, H, W] (= [B, 1, D, H, W]), in_dtype WW_DTYPE_HALF or
 *        WW_DTYPE_FLOAT, finite values; D >= 1
 * out  : [B, 1, H, W], out_dtype WW_DTYPE_HALF or WW_DTYPE_FLOAT
 * fp32 arithmetic: within 1e-5 relative (of max(|disp|, 1)) of the exact
 * value; an fp16 output is that value rounded to nearest.
 * ------------------------------------------------------------------------- */
int ww_disparity_regression(const void* cost, void* out, int in_dtype, int out_dtype, int B, int D, int H, int W,
                            int mode, void* stream);

/* BatchNorm folding on the host: w16[o, :] = fp16(w[o, :] * scale[o]) computed in
 * fp32, b16[o] = fp16(bias[o]); k = Cin * 27.  Host memory only. */
int ww_fold_bn_f16(const float* w, const float* scale, const float* bias, int cout, int k,
                   uint16_t* w16, uint16_t* b16);

/* ---------------------------------------------------------------------------
 * Plugin layer without TensorRT.  These carry the logic of the reference
 * IPluginV3 methods so that the TensorRT shim (csrc/trt/) is a thin
 * forwarder and so the logic is testable without TensorRT.
 * ------------------------------------------------------------------------- */
typedef struct ww_tensor_desc {
    int32_t nb_dims;
    int64_t dims[8];
    int32_t dtype;  /* ww_dtype_t */
    int32_t format; /* WW_FORMAT_LINEAR */
} ww_tensor_desc_t;

/* Creator field parsing (plugin_fields.hpp:17-31 semantics): returns the int
 * value of field `name` among `nb_fields` (names[i], values[i] may be NULL
 * meaning "absent / no data"), else `fallback`. */
int ww_plugin_get_int_field(int nb_fields, const char* const* names, const int32_t* const* values,
                            const char* name, int fallback);

/* "CorrVolume" v"1": field max_disp (default 48) and extension field
 * num_groups (default 1).  Output [B, max_disp, H, W] (num_groups == 1) or
 * [B, num_groups, max_disp, H, W].  corr_volume.cpp:28-82, 113-139. */
int ww_plugin_corr_volume_output_dtype(int nb_inputs, const int32_t* in_dtypes, int32_t* out_dtype);
int ww_plugin_corr_volume_output_dims(int max_disp, int num_groups, int nb_inputs,
                                      const ww_tensor_desc_t* inputs, ww_tensor_desc_t* out);
int ww_plugin_corr_volume_supports_format(int pos, const ww_tensor_desc_t* in_out,
                                          int nb_inputs, int nb_outputs);
/* corr_volume.cpp:84-111: 0 on success, 1 on bad rank, dtype or launch. */
int ww_plugin_corr_volume_enqueue(int max_disp, int num_groups, const ww_tensor_desc_t* in_desc,
                                  const void* const* inputs, void* const* outputs, void* stream);

/* "CostStem3D" v"1": no fields in the reference; 7 inputs (reference) or 3
 * inputs (generalised extension: vol, w, b, with `act` from the optional
 * extension field "act", default 0 = ReLU; ignored for 7 inputs).  Output
 * shape = input 0 shape for 7 inputs, [B, Cout, D, H, W] for 3.
 * cost_stem_3d.cpp:19-73. */
int ww_plugin_cost_stem3d_output_dims(int nb_inputs, const ww_tensor_desc_t* inputs,
                                      ww_tensor_desc_t* out);
int ww_plugin_cost_stem3d_supports_format(int pos, const ww_tensor_desc_t* in_out,
                                          int nb_inputs, int nb_outputs);
int ww_plugin_cost_stem3d_enqueue(int nb_inputs, int act, const ww_tensor_desc_t* in_desc,
                                  const void* const* inputs, void* const* outputs, void* stream);

/* "CorrCostStem3D" v"1" (extension): fields max_disp (48), num_groups (1),
 * act (0 ReLU, 1 ReLU6); inputs left, right [B,C,H,W], w [Cout,G,3,3,3], b [Cout];
 * output [B, Cout, max_disp, H, W]; fp16 only.  output_dims returns 1 for a
 * shape outside ww_corr_cost_stem3d_supported (so an engine build fails,
 * not the enqueue) and when the weights' group count is not num_groups.  With 8 inputs (left, right,
 * w0, b0, w1, b1, w2, b2; num_groups 1) it is ww_corr_cost_stem3d_ref3 and
 * the output is [B, 1, max_disp, H, W]. */
int ww_plugin_corr_cost_stem3d_output_dims(int max_disp, int num_groups, int nb_inputs,
                                           const ww_tensor_desc_t* inputs, ww_tensor_desc_t* out);
int ww_plugin_corr_cost_stem3d_supports_format(int pos, const ww_tensor_desc_t* in_out,
                                               int nb_inputs, int nb_outputs);
/* nb_inputs selects the form: 4 (left, right, w, b) or 8 (left, right, w0,
 * b0, w1, b1, w2, b2).  Every input must be fp16; input 1 must have input 0's
 * shape; the weights and biases must have the element counts of their form. */
int ww_plugin_corr_cost_stem3d_enqueue(int nb_inputs, int max_disp, int num_groups, int act,
                                       const ww_tensor_desc_t* in_desc,
                                       const void* const* inputs, void* const* outputs,
                                       void* stream);

/* "Nv12Decode" v"1": fields out_h (default 224), out_w (default 288); input
 * [B, H_IN * 3 / 2, W_IN] declared INT8 (uint8 bytes), output [B, 3, out_h,
 * out_w] declared FLOAT, built as fp16 or fp32.  nv12_decode.cpp:26-146. */
int ww_plugin_nv12_decode_output_dtype(int nb_inputs, int32_t* out_dtype);
int ww_plugin_nv12_decode_output_dims(int out_h, int out_w, int nb_inputs, const ww_tensor_desc_t* inputs,
                                      ww_tensor_desc_t* out);
int ww_plugin_nv12_decode_supports_format(int pos, const ww_tensor_desc_t* in_out, int nb_inputs,
                                          int nb_outputs);
int ww_plugin_nv12_decode_enqueue(int out_h, int out_w, const ww_tensor_desc_t* in_desc,
                                  const ww_tensor_desc_t* out_desc, const void* const* inputs,
                                  void* const* outputs, void* stream);

/* "DisparityRegression" v"1" (extension; no reference counterpart): field
 * mode (0 soft-argmax, 1 soft-argmin; default 0); input cost [B, D, H, W] or
 * [B, 1, D, H, W] fp16 or fp32; output [B, 1, H, W], same dtype as the
 * input. */
int ww_plugin_disparity_regression_output_dims(int nb_inputs, const ww_tensor_desc_t* inputs,
                                               ww_tensor_desc_t* out);
int ww_plugin_disparity_regression_supports_format(int pos, const ww_tensor_desc_t* in_out, int nb_inputs,
                                                   int nb_outputs);
int ww_plugin_disparity_regression_enqueue(int mode, const ww_tensor_desc_t* in_desc,
                                           const ww_tensor_desc_t* out_desc, const void* const* inputs,
                                           void* const* outputs, void* stream);

/* Device error word written by bounded waits inside the tensor-core kernels
 * (0 = none).  There is ONE word per device, shared by every call, stream and
 * thread that uses the device: the first wait that expires in any launch
 * records its code there, and the word keeps it (later expiries do not
 * overwrite it) until ww_clear_device_error() resets it to 0.  So a non-zero
 * value says that some launch on the device since the last clear gave up a
 * wait, not which one; a caller that needs to attribute it clears the word,
 * runs the call alone and reads it after the call has completed.  Reading
 * synchronises the current device; clearing is a blocking device write. */
int ww_device_error(int* code);
int ww_clear_device_error(void);

#ifdef __cplusplus
}
#endif
#endif /* WW_TRT_PLUGINS_H */

/*
 * ww_oracle.h -- scalar CPU restatement of the stereo cost-volume front end.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * CUDA path in whirlwind_trt_plugins_b200/.  Only tests/, the smoke check in
 * __graft_entry__.py and the cpu_baseline / reference arm of bench.py may
 * load it.  The product never calls it and has no CPU fallback.
 *
 * Parity pinning: the oracle is checked bit-for-bit against the reference's
 * own CUDA kernels (corr_volume_kernel.cu, cost_stem_3d_kernel.cu rebuilt
 * for sm_100a from the unmodified reference sources by oracle/Makefile) via
 * the golden fixtures in tests/golden/, generated on a B200 by
 * tests/golden/make_golden.py.  The reference ships no test vectors of its
 * own, so those fixtures are the pin.
 *
 * Every function cites the reference file:line whose semantics it restates
 * (paths relative to the reference project root).
 *
 * Tensor layouts (all row-major, "NCHW"/"NCDHW"):
 *   left/right    [B, C, H, W]
 *   cost volume   [B, G, D, H, W]        (G == 1 is the reference [B, D, H, W])
 *   stem weights  [Cout, Cin, 3, 3, 3]   (OIDHW, as the reference indexes them)
 *   stem output   [B, Cout, D, H, W]
 * fp16 tensors are passed as uint16_t bit patterns.
 */
#ifndef WW_ORACLE_H
#define WW_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* How the channel mean is formed after the fp32 sum (see orc_corr_f16).   */
enum {
    ORC_SCALE_DIV = 0,    /* acc / (float)C      corr_volume_kernel.cu:84   */
    ORC_SCALE_MULINV = 1  /* acc * (1.0f / C)    corr_volume_kernel.cu:227,356 */
};

/* Accumulation mode of the generalised stem. */
enum {
    ORC_ACC_F32_SEQ = 0,  /* fmaf in (ci, kd, kh, kw) order, like cost_stem_3d_kernel.cu:164-179 */
    ORC_ACC_F64 = 1       /* double accumulation, one rounding at the end ("truth") */
};

enum { ORC_ACT_RELU = 0, ORC_ACT_RELU6 = 1 };

/* IEEE binary16 <-> binary32, round-to-nearest-even, own implementation. */
uint16_t orc_f32_to_f16(float f);
float orc_f16_to_f32(uint16_t h);
void orc_f32_to_f16_array(const float* src, uint16_t* dst, int64_t n);
void orc_f16_to_f32_array(const uint16_t* src, float* dst, int64_t n);

/* Which of the reference's two CorrVolume kernels launchCorrVolume<__half>
 * would pick for one call (corr_volume_kernel.cu:333-368): returns
 * ORC_SCALE_MULINV when corrVolumeFastKernel runs, ORC_SCALE_DIV when the
 * naive corrVolumeKernel runs.  Restates fastPathApplies/pickTileW
 * (corr_volume_kernel.cu:251-326) for an SM count `sm_count`.          */
int orc_ref_corr_scale_mode(int is_half, int B, int C, int H, int W, int D, int sm_count);

/* Correlation volume (corr_volume_kernel.cu:52-88 and :118-239), group-wise:
 *   out[b,g,d,h,w] = scale( sum_{c in group g} L[b,c,h,w] * R[b,c,h,w-d] )
 * with the sum a sequential fp32 fma chain over c (what nvcc emits for
 * `acc += a*b`), scale per `scale_mode`, and exact +0 when w-d < 0.
 * G must divide C.  `nthreads` <= 0 uses all hardware threads.          */
int orc_corr_f32(const float* L, const float* R, float* out,
                 int B, int C, int H, int W, int D, int G, int nthreads);
int orc_corr_f16(const uint16_t* L, const uint16_t* R, uint16_t* out,
                 int B, int C, int H, int W, int D, int G, int scale_mode, int nthreads);

/* The reference's fused 3-stage stem (cost_stem_3d_kernel.cu:71-233):
 * three Conv3d 3x3x3 pad 1 (1->4->4->1) + bias + ReLU6 with fp16 rounding
 * between stages, restated layer by layer with per-layer zero padding.
 * Unlike the reference kernel (which only ever writes batch 0,
 * cost_stem_3d_kernel.cu:92) every batch item is computed.             */
int orc_stem_ref3(const uint16_t* in, uint16_t* out,
                  const uint16_t* w0, const uint16_t* b0,
                  const uint16_t* w1, const uint16_t* b1,
                  const uint16_t* w2, const uint16_t* b2,
                  int B, int D, int H, int W, int nthreads);

/* Generalised single-layer stem: Conv3d 3x3x3 pad 1, Cin -> Cout, folded-BN
 * bias, ReLU or ReLU6, fp16 out.  Output rows [h0, h1) of batch items
 * [b0, b1) only (pass 0,B / 0,H for the whole tensor); `out` is always the
 * full [B, Cout, D, H, W] tensor and other rows are left untouched.    */
int orc_stem(const uint16_t* vol, const uint16_t* w, const uint16_t* bias, uint16_t* out,
             int B, int Cin, int Cout, int D, int H, int W, int act, int acc_mode,
             int b0, int b1, int h0, int h1, int nthreads);

/* Fused front end: correlation (fp16 volume, `scale_mode`) then the
 * generalised stem over G groups -> Cout.  Only output rows [h0, h1) of
 * batch items [b0, b1) are produced; the volume rows they need
 * ([h0-1, h1+1)) are computed internally, never for the whole tensor.  */
int orc_corr_stem(const uint16_t* L, const uint16_t* R, const uint16_t* w, const uint16_t* bias,
                  uint16_t* out, int B, int C, int G, int H, int W, int D, int Cout,
                  int act, int scale_mode, int acc_mode,
                  int b0, int b1, int h0, int h1, int nthreads);

/* Folded BatchNorm: w16[o,:] = f16(w[o,:] * scale[o]) computed in fp32,
 * b16[o] = f16(bias[o]).  `k` = Cin * 27.                              */
void orc_fold_bn(const float* w, const float* scale, const float* bias,
                 int cout, int k, uint16_t* w16, uint16_t* b16);

int orc_hw_threads(void);

/* NV12 [B, H_IN * 3 / 2, W_IN] uint8 -> planar RGB [B, 3, H_OUT, W_OUT] in
 * [-1, 1] (fp16 bit patterns if out_f16, else fp32): bilinear resize with
 * align_corners = False and clamped taps, full-range BT.601 fused with
 * 2 * (rgb / 255) - 1 (nv12_decode_kernel.cu:33-188, launcher :197-230).
 * Every batch item (the reference plugin decodes batch 0 only).         */
int orc_nv12_decode(const uint8_t* nv12, int B, int H_IN, int W_IN, int H_OUT, int W_OUT, int out_f16,
                    void* out, int nthreads);

/* Disparity regression, the step after the 3-D aggregation (no reference
 * counterpart; this formula is its specification):
 *   disp[b, h, w] = sum_d d * softmax_d(s * cost[b, d, h, w]),
 * s = +1 (mode 0, soft-argmax) or -1 (mode 1, soft-argmin); cost [B, D, H, W]
 * fp16 bit patterns if in_f16, else fp32; evaluated in double and rounded
 * once to the output type (fp16 bit patterns if out_f16, else fp32).     */
int orc_disparity_regression(const void* cost, int in_f16, int B, int D, int H, int W, int mode, int out_f16,
                             void* out, int nthreads);

#ifdef __cplusplus
}
#endif
#endif

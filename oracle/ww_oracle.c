/*
 * ww_oracle.c -- scalar CPU restatement of the reference's CorrVolume and
 * CostStem3D semantics plus the group-wise / generalised-stem extension.
 *
 * TEST INFRASTRUCTURE ONLY (see ww_oracle.h): the parity checker and the
 * CPU baseline, never part of the product path.
 *
 * Arithmetic follows the reference kernels operation for operation where
 * the reference defines it:
 *   - correlation: one fp32 fma chain over the channels of a group, in
 *     channel order, starting from +0 (corr_volume_kernel.cu:73-82 and
 *     :211-216; nvcc contracts `acc += a*b` into fma), then either a true
 *     division by C (naive kernel, :84) or a multiply by the host-computed
 *     1.0f/C (fast kernel, :227 with invC from :356), rounded to fp16 RNE;
 *     +0 wherever w - d < 0 (:75 / the zero-staged halo at :179-186).
 *   - reference stem: per stage an fma chain in (ci, kd, kh, kw) order,
 *     then + bias, ReLU6, fp16 RNE; positions outside the volume are zero
 *     for the next stage (cost_stem_3d_kernel.cu:115-232).
 *
 *   - disparity regression has no reference counterpart: it is evaluated
 *     from its formula in double (no parity pin exists for it).
 *
 * Skipping a zero-padding tap is bit-identical to multiplying the staged
 * zero the reference multiplies: the accumulator starts at +0 and an RNE
 * fma chain never produces -0 from a +0 start, so acc + (+-0) == acc.
 */
#define _GNU_SOURCE
#include "ww_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------------ */
/* fp16 conversion                                                     */
/* ------------------------------------------------------------------ */

/* Round a double to the nearest binary16 (ties to even).  Scaling by a
 * power of two is exact in double, so nearbyint() performs the single
 * correct rounding.  A float argument converts to double exactly, so this
 * is also the correctly rounded float -> half conversion.              */
static uint16_t half_from_double(double x)
{
    uint16_t sign = signbit(x) ? 0x8000u : 0u;
    double ax = fabs(x);
    if (isnan(x)) return (uint16_t)(sign | 0x7e00u);
    if (ax >= 65520.0) return (uint16_t)(sign | 0x7c00u); /* rounds to inf */
    if (ax < 6.103515625e-05) {                           /* < 2^-14: subnormal range */
        double m = nearbyint(ldexp(ax, 24));              /* units of 2^-24 */
        return (uint16_t)(sign | (uint16_t)m);            /* m == 1024 is min normal */
    }
    int ex;
    (void)frexp(ax, &ex);                                 /* ax = f * 2^ex, f in [0.5,1) */
    int e = ex - 1;                                       /* ax in [2^e, 2^(e+1)) */
    double m = nearbyint(ldexp(ax, 10 - e));              /* in [1024, 2048] */
    if (m >= 2048.0) { m = 1024.0; e += 1; }
    int field = e + 15;
    if (field >= 31) return (uint16_t)(sign | 0x7c00u);
    return (uint16_t)(sign | (uint16_t)(field << 10) | (uint16_t)((int)m - 1024));
}

uint16_t orc_f32_to_f16(float f) { return half_from_double((double)f); }

float orc_f16_to_f32(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x3ffu;
    float v;
    if (exp == 0) {
        v = (float)mant * 5.9604644775390625e-08f; /* mant * 2^-24, exact */
        uint32_t bits;
        memcpy(&bits, &v, 4);
        bits |= sign;
        memcpy(&v, &bits, 4);
        return v;
    }
    uint32_t bits;
    if (exp == 31) bits = sign | 0x7f800000u | (mant << 13);
    else bits = sign | ((exp + 112u) << 23) | (mant << 13);
    memcpy(&v, &bits, 4);
    return v;
}

void orc_f32_to_f16_array(const float* src, uint16_t* dst, int64_t n)
{
    for (int64_t i = 0; i < n; ++i) dst[i] = orc_f32_to_f16(src[i]);
}

void orc_f16_to_f32_array(const uint16_t* src, float* dst, int64_t n)
{
    for (int64_t i = 0; i < n; ++i) dst[i] = orc_f16_to_f32(src[i]);
}

/* ------------------------------------------------------------------ */
/* Thread pool: a parallel-for over [0, n) with an atomic work counter  */
/* ------------------------------------------------------------------ */

int orc_hw_threads(void)
{
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

typedef void (*orc_body_fn)(void* ctx, int64_t i);

typedef struct {
    orc_body_fn fn;
    void* ctx;
    int64_t n;
    int64_t next;
    pthread_mutex_t mu;
} orc_pool_t;

static void* orc_worker(void* arg)
{
    orc_pool_t* p = (orc_pool_t*)arg;
    for (;;) {
        pthread_mutex_lock(&p->mu);
        int64_t i = p->next++;
        pthread_mutex_unlock(&p->mu);
        if (i >= p->n) break;
        p->fn(p->ctx, i);
    }
    return NULL;
}

static void orc_parallel_for(int64_t n, int nthreads, orc_body_fn fn, void* ctx)
{
    if (nthreads <= 0) nthreads = orc_hw_threads();
    if (nthreads > n) nthreads = (int)(n > 0 ? n : 1);
    orc_pool_t pool;
    pool.fn = fn;
    pool.ctx = ctx;
    pool.n = n;
    pool.next = 0;
    pthread_mutex_init(&pool.mu, NULL);
    if (nthreads <= 1) {
        orc_worker(&pool);
    } else {
        pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nthreads);
        int started = 0;
        for (int t = 0; t < nthreads; ++t)
            if (pthread_create(&th[t], NULL, orc_worker, &pool) == 0) ++started;
        if (started == 0) orc_worker(&pool);
        for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
        free(th);
    }
    pthread_mutex_destroy(&pool.mu);
}

/* ------------------------------------------------------------------ */
/* Reference kernel selection (corr_volume_kernel.cu:251-368)          */
/* ------------------------------------------------------------------ */

static int round_up(int v, int m) { return (v + m - 1) / m * m; }

/* pickTileW, corr_volume_kernel.cu:251-312: full-row tile, split for
 * occupancy when H*B < SMs/2, capped by 48 KB of shared memory and 1024
 * threads, rounded to 8, then balanced.                                */
static int ref_pick_tile(int C, int B, int H, int W, int PADA, int dispY, int sm_count)
{
    const int kMinTileW = 32, kSmemLimit = 48 * 1024, kVecW = 4;
    int tile = round_up(W, 8);
    const int rowBlocks = H * B;
    const int target = sm_count / 2;
    if (rowBlocks > 0 && rowBlocks < target && tile > 2 * kMinTileW) {
        const int wantSplit = (target + rowBlocks - 1) / rowBlocks;
        const int split = round_up((W + wantSplit - 1) / wantSplit, 8);
        if (split > 0 && split < tile) tile = split;
        if (tile < kMinTileW) tile = kMinTileW;
    }
    const int byBytes = (kSmemLimit / (2 * C) - PADA) / 2;
    if (tile > byBytes) tile = byBytes;
    const int byThreads = 1024 / dispY * kVecW;
    if (tile > byThreads) tile = byThreads;
    tile = tile / 8 * 8;
    if (tile < 8) return 0;
    const int gridX = (W + tile - 1) / tile;
    if (gridX > 1) {
        const int balanced = round_up((W + gridX - 1) / gridX, 8);
        if (balanced >= kMinTileW && balanced < tile) tile = balanced;
    }
    return tile;
}

int orc_ref_corr_scale_mode(int is_half, int B, int C, int H, int W, int D, int sm_count)
{
    /* launchCorrVolume<float> always runs the naive kernel (:373 is
     * half-only); the naive kernel divides.                            */
    if (!is_half) return ORC_SCALE_DIV;
    if (D <= 0 || D % 6 != 0) return ORC_SCALE_DIV;
    const int dispY = D / 6;
    const int PADA = round_up(D - 1, 8);
    const int tile = ref_pick_tile(C, B, H, W, PADA, dispY, sm_count);
    /* fastPathApplies, corr_volume_kernel.cu:314-326 */
    if (W % 8 != 0) return ORC_SCALE_DIV;
    const long long outputs = (long long)B * D * H * W;
    if (outputs < (long long)sm_count * 800) return ORC_SCALE_DIV;
    if (tile < 8 || tile % 8 != 0) return ORC_SCALE_DIV;
    const long long smem = (long long)C * (tile + tile + PADA) * 2;
    if (smem > 48 * 1024) return ORC_SCALE_DIV;
    const int threads = (tile / 4) * dispY;
    if (threads <= 0 || threads > 1024) return ORC_SCALE_DIV;
    return ORC_SCALE_MULINV;
}

/* ------------------------------------------------------------------ */
/* Correlation                                                          */
/* ------------------------------------------------------------------ */

typedef struct {
    const float* L;
    const float* R;
    void* out;
    int is_half;
    int B, C, H, W, D, G;
    int scale_mode;
    int h0, h1;           /* rows computed                          */
    int out_h0, out_rows; /* out is [B?][G][D][out_rows][W] at row offset out_h0 */
    int64_t out_bstride;  /* elements between batch items of out   */
    int b0;
} corr_ctx_t;

/* One work item = (b, g, d): rows [h0, h1) x all W. */
static void corr_body(void* vctx, int64_t item)
{
    const corr_ctx_t* k = (const corr_ctx_t*)vctx;
    const int D = k->D, G = k->G, H = k->H, W = k->W, C = k->C;
    const int Cg = C / G;
    const int d = (int)(item % D);
    const int g = (int)((item / D) % G);
    const int b = k->b0 + (int)(item / ((int64_t)D * G));
    const float invC = 1.0f / (float)Cg;
    float* acc = (float*)malloc(sizeof(float) * (size_t)(W > 0 ? W : 1));
    for (int h = k->h0; h < k->h1; ++h) {
        for (int w = 0; w < W; ++w) acc[w] = 0.0f;
        for (int c = g * Cg; c < (g + 1) * Cg; ++c) {
            const float* lrow = k->L + (((int64_t)b * C + c) * H + h) * W;
            const float* rrow = k->R + (((int64_t)b * C + c) * H + h) * W;
            for (int w = d; w < W; ++w) acc[w] = fmaf(lrow[w], rrow[w - d], acc[w]);
        }
        const int64_t obase = (int64_t)(b - k->b0) * k->out_bstride +
                              (((int64_t)g * D + d) * k->out_rows + (h - k->out_h0)) * W;
        for (int w = 0; w < W; ++w) {
            float v;
            if (w < d) v = 0.0f;
            else if (k->scale_mode == ORC_SCALE_DIV) v = acc[w] / (float)Cg;
            else v = acc[w] * invC;
            if (k->is_half) ((uint16_t*)k->out)[obase + w] = orc_f32_to_f16(v);
            else ((float*)k->out)[obase + w] = v;
        }
    }
    free(acc);
}

static int corr_args_ok(int B, int C, int H, int W, int D, int G)
{
    return B >= 0 && C > 0 && H >= 0 && W >= 0 && D >= 0 && G > 0 && C % G == 0;
}

int orc_corr_f32(const float* L, const float* R, float* out,
                 int B, int C, int H, int W, int D, int G, int nthreads)
{
    if (!corr_args_ok(B, C, H, W, D, G)) return 1;
    corr_ctx_t k = {L, R, out, 0, B, C, H, W, D, G, ORC_SCALE_DIV, 0, H, 0, H,
                    (int64_t)G * D * H * W, 0};
    orc_parallel_for((int64_t)B * G * D, nthreads, corr_body, &k);
    return 0;
}

static float* widen_half(const uint16_t* src, int64_t n)
{
    float* f = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    if (f) orc_f16_to_f32_array(src, f, n);
    return f;
}

int orc_corr_f16(const uint16_t* L, const uint16_t* R, uint16_t* out,
                 int B, int C, int H, int W, int D, int G, int scale_mode, int nthreads)
{
    if (!corr_args_ok(B, C, H, W, D, G)) return 1;
    const int64_t n = (int64_t)B * C * H * W;
    float* Lf = widen_half(L, n);
    float* Rf = widen_half(R, n);
    if (!Lf || !Rf) { free(Lf); free(Rf); return 2; }
    corr_ctx_t k = {Lf, Rf, out, 1, B, C, H, W, D, G, scale_mode, 0, H, 0, H,
                    (int64_t)G * D * H * W, 0};
    orc_parallel_for((int64_t)B * G * D, nthreads, corr_body, &k);
    free(Lf);
    free(Rf);
    return 0;
}

/* ------------------------------------------------------------------ */
/* Reference 3-stage stem (cost_stem_3d_kernel.cu:71-233)               */
/* ------------------------------------------------------------------ */

static float relu6f(float v) { return fminf(6.0f, fmaxf(0.0f, v)); }

/* One Conv3d 3x3x3 pad-1 stage over fp16-valued float inputs
 * src[cin][D][H][W] -> dst[cout][D][H][W] (rounded to fp16 values),
 * accumulation order (ci, kd, kh, kw) as at cost_stem_3d_kernel.cu:164-179. */
static void ref3_stage(const float* src, float* dst, const float* wt, const float* bias,
                       int cin, int cout, int D, int H, int W)
{
    for (int co = 0; co < cout; ++co)
        for (int d = 0; d < D; ++d)
            for (int h = 0; h < H; ++h)
                for (int w = 0; w < W; ++w) {
                    float acc = 0.0f;
                    for (int ci = 0; ci < cin; ++ci)
                        for (int kd = 0; kd < 3; ++kd)
                            for (int kh = 0; kh < 3; ++kh)
                                for (int kw = 0; kw < 3; ++kw) {
                                    const int sd = d + kd - 1, sh = h + kh - 1, sw = w + kw - 1;
                                    float v = 0.0f;
                                    if (sd >= 0 && sd < D && sh >= 0 && sh < H && sw >= 0 && sw < W)
                                        v = src[(((int64_t)ci * D + sd) * H + sh) * W + sw];
                                    acc = fmaf(v, wt[((co * cin + ci) * 3 + kd) * 9 + kh * 3 + kw], acc);
                                }
                    acc += bias[co];
                    dst[(((int64_t)co * D + d) * H + h) * W + w] =
                        orc_f16_to_f32(orc_f32_to_f16(relu6f(acc)));
                }
}

typedef struct {
    const uint16_t* in;
    uint16_t* out;
    float wf0[108], bf0[4], wf1[432], bf1[4], wf2[108], bf2[1];
    int D, H, W;
} ref3_ctx_t;

static void ref3_body(void* vctx, int64_t b)
{
    const ref3_ctx_t* k = (const ref3_ctx_t*)vctx;
    const int64_t vol = (int64_t)k->D * k->H * k->W;
    float* x = (float*)malloc(sizeof(float) * (size_t)(vol > 0 ? vol : 1));
    float* s0 = (float*)malloc(sizeof(float) * (size_t)(4 * vol > 0 ? 4 * vol : 1));
    float* s1 = (float*)malloc(sizeof(float) * (size_t)(4 * vol > 0 ? 4 * vol : 1));
    float* s2 = (float*)malloc(sizeof(float) * (size_t)(vol > 0 ? vol : 1));
    orc_f16_to_f32_array(k->in + b * vol, x, vol);
    ref3_stage(x, s0, k->wf0, k->bf0, 1, 4, k->D, k->H, k->W);
    ref3_stage(s0, s1, k->wf1, k->bf1, 4, 4, k->D, k->H, k->W);
    ref3_stage(s1, s2, k->wf2, k->bf2, 4, 1, k->D, k->H, k->W);
    orc_f32_to_f16_array(s2, k->out + b * vol, vol);
    free(x);
    free(s0);
    free(s1);
    free(s2);
}

int orc_stem_ref3(const uint16_t* in, uint16_t* out,
                  const uint16_t* w0, const uint16_t* b0,
                  const uint16_t* w1, const uint16_t* b1,
                  const uint16_t* w2, const uint16_t* b2,
                  int B, int D, int H, int W, int nthreads)
{
    if (B < 0 || D < 0 || H < 0 || W < 0) return 1;
    ref3_ctx_t* k = (ref3_ctx_t*)malloc(sizeof(ref3_ctx_t));
    if (!k) return 2;
    k->in = in;
    k->out = out;
    k->D = D;
    k->H = H;
    k->W = W;
    orc_f16_to_f32_array(w0, k->wf0, 108);
    orc_f16_to_f32_array(b0, k->bf0, 4);
    orc_f16_to_f32_array(w1, k->wf1, 432);
    orc_f16_to_f32_array(b1, k->bf1, 4);
    orc_f16_to_f32_array(w2, k->wf2, 108);
    orc_f16_to_f32_array(b2, k->bf2, 1);
    orc_parallel_for(B, nthreads, ref3_body, k);
    free(k);
    return 0;
}

/* ------------------------------------------------------------------ */
/* Generalised stem: Conv3d 3x3x3 pad 1, Cin -> Cout, bias, ReLU/ReLU6  */
/* ------------------------------------------------------------------ */

typedef struct {
    const float* volf;   /* [nb][Cin][D][Hv][W] fp16 values as float   */
    int64_t vol_bstride; /* elements between batch items of volf       */
    int hv0, Hv;         /* volf row r holds global row hv0 + r         */
    const float* wf;     /* [Cout][Cin][27]                             */
    const float* bf;     /* [Cout]                                      */
    uint16_t* out;       /* [B][Cout][D][H][W]                          */
    int b0, Cin, Cout, D, H, W, act, acc_mode, h0, h1;
} stem_ctx_t;

static float act_apply(float v, int act) { return act == ORC_ACT_RELU6 ? relu6f(v) : fmaxf(0.0f, v); }

/* One work item = (b, o, d): output rows [h0, h1) x all W. */
static void stem_body(void* vctx, int64_t item)
{
    const stem_ctx_t* k = (const stem_ctx_t*)vctx;
    const int D = k->D, H = k->H, W = k->W, Cin = k->Cin, Cout = k->Cout;
    const int d = (int)(item % D);
    const int o = (int)((item / D) % Cout);
    const int bl = (int)(item / ((int64_t)D * Cout));
    const int b = k->b0 + bl;
    const float* vb = k->volf + (int64_t)bl * k->vol_bstride;
    float* accf = (float*)malloc(sizeof(float) * (size_t)(W > 0 ? W : 1));
    double* accd = (double*)malloc(sizeof(double) * (size_t)(W > 0 ? W : 1));
    for (int h = k->h0; h < k->h1; ++h) {
        for (int w = 0; w < W; ++w) { accf[w] = 0.0f; accd[w] = 0.0; }
        for (int ci = 0; ci < Cin; ++ci)
            for (int kd = 0; kd < 3; ++kd) {
                const int sd = d + kd - 1;
                if (sd < 0 || sd >= D) continue;
                for (int kh = 0; kh < 3; ++kh) {
                    const int sh = h + kh - 1;
                    if (sh < 0 || sh >= H) continue;
                    const int r = sh - k->hv0;
                    const float* row = vb + (((int64_t)ci * D + sd) * k->Hv + r) * W;
                    for (int kw = 0; kw < 3; ++kw) {
                        const float wt = k->wf[((int64_t)o * Cin + ci) * 27 + kd * 9 + kh * 3 + kw];
                        const int lo = kw == 0 ? 1 : 0;          /* w + kw - 1 >= 0 */
                        const int hi = kw == 2 ? W - 1 : W;      /* w + kw - 1 <  W */
                        if (k->acc_mode == ORC_ACC_F64) {
                            for (int w = lo; w < hi; ++w) accd[w] += (double)row[w + kw - 1] * (double)wt;
                        } else {
                            for (int w = lo; w < hi; ++w) accf[w] = fmaf(row[w + kw - 1], wt, accf[w]);
                        }
                    }
                }
            }
        uint16_t* orow = k->out + ((((int64_t)b * Cout + o) * D + d) * H + h) * W;
        for (int w = 0; w < W; ++w) {
            if (k->acc_mode == ORC_ACC_F64) {
                double v = accd[w] + (double)k->bf[o];
                v = k->act == ORC_ACT_RELU6 ? fmin(6.0, fmax(0.0, v)) : fmax(0.0, v);
                orow[w] = half_from_double(v);
            } else {
                orow[w] = orc_f32_to_f16(act_apply(accf[w] + k->bf[o], k->act));
            }
        }
    }
    free(accf);
    free(accd);
}

static int stem_args_ok(int B, int Cin, int Cout, int D, int H, int W, int b0, int b1, int h0, int h1)
{
    return B >= 0 && Cin > 0 && Cout > 0 && D >= 0 && H >= 0 && W >= 0 &&
           0 <= b0 && b0 <= b1 && b1 <= B && 0 <= h0 && h0 <= h1 && h1 <= H;
}

int orc_stem(const uint16_t* vol, const uint16_t* w, const uint16_t* bias, uint16_t* out,
             int B, int Cin, int Cout, int D, int H, int W, int act, int acc_mode,
             int b0, int b1, int h0, int h1, int nthreads)
{
    if (!stem_args_ok(B, Cin, Cout, D, H, W, b0, b1, h0, h1)) return 1;
    const int64_t per_b = (int64_t)Cin * D * H * W;
    float* volf = widen_half(vol + (int64_t)b0 * per_b, (int64_t)(b1 - b0) * per_b);
    float* wf = widen_half(w, (int64_t)Cout * Cin * 27);
    float* bf = widen_half(bias, Cout);
    if (!volf || !wf || !bf) { free(volf); free(wf); free(bf); return 2; }
    stem_ctx_t k = {volf, per_b, 0, H, wf, bf, out, b0, Cin, Cout, D, H, W, act, acc_mode, h0, h1};
    orc_parallel_for((int64_t)(b1 - b0) * Cout * D, nthreads, stem_body, &k);
    free(volf);
    free(wf);
    free(bf);
    return 0;
}

int orc_corr_stem(const uint16_t* L, const uint16_t* R, const uint16_t* w, const uint16_t* bias,
                  uint16_t* out, int B, int C, int G, int H, int W, int D, int Cout,
                  int act, int scale_mode, int acc_mode,
                  int b0, int b1, int h0, int h1, int nthreads)
{
    if (!corr_args_ok(B, C, H, W, D, G)) return 1;
    if (!stem_args_ok(B, G, Cout, D, H, W, b0, b1, h0, h1)) return 1;
    if (b1 == b0 || h1 == h0) return 0;
    /* Volume rows needed by output rows [h0, h1): [h0-1, h1+1) clipped. */
    const int hv0 = h0 > 0 ? h0 - 1 : 0;
    const int hv1 = h1 < H ? h1 + 1 : H;
    const int Hv = hv1 - hv0;
    const int nb = b1 - b0;
    const int64_t in_per_b = (int64_t)C * H * W;
    float* Lf = widen_half(L + (int64_t)b0 * in_per_b, (int64_t)nb * in_per_b);
    float* Rf = widen_half(R + (int64_t)b0 * in_per_b, (int64_t)nb * in_per_b);
    const int64_t vol_per_b = (int64_t)G * D * Hv * W;
    uint16_t* vol16 = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(nb * vol_per_b > 0 ? nb * vol_per_b : 1));
    if (!Lf || !Rf || !vol16) { free(Lf); free(Rf); free(vol16); return 2; }
    /* Lf/Rf hold batch items [b0, b1) re-based at 0. */
    corr_ctx_t kc = {Lf, Rf, vol16, 1, nb, C, H, W, D, G, scale_mode, hv0, hv1, hv0, Hv,
                     vol_per_b, 0};
    orc_parallel_for((int64_t)nb * G * D, nthreads, corr_body, &kc);
    free(Lf);
    free(Rf);
    float* volf = widen_half(vol16, nb * vol_per_b);
    free(vol16);
    float* wf = widen_half(w, (int64_t)Cout * G * 27);
    float* bf = widen_half(bias, Cout);
    if (!volf || !wf || !bf) { free(volf); free(wf); free(bf); return 2; }
    stem_ctx_t ks = {volf, vol_per_b, hv0, Hv, wf, bf, out, b0, G, Cout, D, H, W, act, acc_mode, h0, h1};
    orc_parallel_for((int64_t)nb * Cout * D, nthreads, stem_body, &ks);
    free(volf);
    free(wf);
    free(bf);
    return 0;
}

void orc_fold_bn(const float* w, const float* scale, const float* bias,
                 int cout, int k, uint16_t* w16, uint16_t* b16)
{
    for (int o = 0; o < cout; ++o) {
        for (int i = 0; i < k; ++i) w16[(int64_t)o * k + i] = orc_f32_to_f16(w[(int64_t)o * k + i] * scale[o]);
        b16[o] = orc_f32_to_f16(bias[o]);
    }
}

/* ------------------------------------------------------------------ */
/* NV12 -> normalised planar RGB (nv12_decode_kernel.cu:33-188)         */
/* ------------------------------------------------------------------ */
/* Per output pixel, in fp32, operation for operation as nvcc compiles the
 * reference expressions (it contracts a*b + c into one fma; both the CUDA
 * kernel of this library and this restatement spell the contractions out):
 *   src = fma(dst + 0.5, scale, -0.5)                       (:130-139)
 *   bilinear: top = fma(wx0, v00, wx1 * v01), bot likewise,
 *             val = fma(wy0, top, wy1 * bot)               (:58, :97-98)
 *   coordinates clamped to the plane after the weights      (:48-51, :78-81)
 *   R = fma(s, fma(1.402, Cr, Y), -1)
 *   G = fma(s, fma(-0.714136, Cr, fma(-0.344136, Cb, Y)), -1)
 *   B = fma(s, fma(1.772, Cb, Y), -1),  s = 2/255, Cb = U - 128, Cr = V - 128
 *                                                           (:104-113, :143)
 * The reference launcher covers batch item 0 only (nv12_decode.cpp:96-114
 * passes no batch to launchNv12Decode); every batch item is computed here. */

static float nv12_bilinear(const uint8_t* plane, int rows, int cols, int row_stride, int step, float yf,
                           float xf)
{
    const int y0 = (int)floorf(yf), x0 = (int)floorf(xf);
    const float wy1 = yf - (float)y0, wy0 = 1.0f - wy1;
    const float wx1 = xf - (float)x0, wx0 = 1.0f - wx1;
    const int y0c = y0 < 0 ? 0 : (y0 > rows - 1 ? rows - 1 : y0);
    const int y1c = y0 + 1 < 0 ? 0 : (y0 + 1 > rows - 1 ? rows - 1 : y0 + 1);
    const int x0c = x0 < 0 ? 0 : (x0 > cols - 1 ? cols - 1 : x0);
    const int x1c = x0 + 1 < 0 ? 0 : (x0 + 1 > cols - 1 ? cols - 1 : x0 + 1);
    const float v00 = (float)plane[(int64_t)y0c * row_stride + (int64_t)step * x0c];
    const float v01 = (float)plane[(int64_t)y0c * row_stride + (int64_t)step * x1c];
    const float v10 = (float)plane[(int64_t)y1c * row_stride + (int64_t)step * x0c];
    const float v11 = (float)plane[(int64_t)y1c * row_stride + (int64_t)step * x1c];
    const float top = fmaf(wx0, v00, wx1 * v01);
    const float bot = fmaf(wx0, v10, wx1 * v11);
    return fmaf(wy0, top, wy1 * bot);
}

typedef struct {
    const uint8_t* nv12;
    int H_IN, W_IN, H_OUT, W_OUT, out_f16;
    void* out;
    float sy_h, sy_w, suv_h, suv_w;
} nv12_ctx;

static void nv12_body(void* vctx, int64_t item)  /* item = b * H_OUT + y */
{
    const nv12_ctx* c = (const nv12_ctx*)vctx;
    const int b = (int)(item / c->H_OUT), y = (int)(item % c->H_OUT);
    const int64_t in_img = (int64_t)c->H_IN * 3 / 2 * c->W_IN;
    const uint8_t* img = c->nv12 + (int64_t)b * in_img;
    const uint8_t* chroma = img + (int64_t)c->H_IN * c->W_IN;
    const int H_UV = c->H_IN >> 1, W_UV = c->W_IN >> 1;
    const int64_t plane = (int64_t)c->H_OUT * c->W_OUT;
    const float s = 2.0f / 255.0f;
    const float yf_y = fmaf((float)y + 0.5f, c->sy_h, -0.5f);
    const float yf_uv = fmaf((float)y + 0.5f, c->suv_h, -0.5f);
    for (int x = 0; x < c->W_OUT; ++x) {
        const float xf_y = fmaf((float)x + 0.5f, c->sy_w, -0.5f);
        const float xf_uv = fmaf((float)x + 0.5f, c->suv_w, -0.5f);
        const float Y = nv12_bilinear(img, c->H_IN, c->W_IN, c->W_IN, 1, yf_y, xf_y);
        const float U = nv12_bilinear(chroma, H_UV, W_UV, c->W_IN, 2, yf_uv, xf_uv);
        const float V = nv12_bilinear(chroma + 1, H_UV, W_UV, c->W_IN, 2, yf_uv, xf_uv);
        const float Cb = U - 128.0f, Cr = V - 128.0f;
        const float R = fmaf(s, fmaf(1.402f, Cr, Y), -1.0f);
        const float G = fmaf(s, fmaf(-0.714136f, Cr, fmaf(-0.344136f, Cb, Y)), -1.0f);
        const float B = fmaf(s, fmaf(1.772f, Cb, Y), -1.0f);
        const int64_t o = ((int64_t)b * 3) * plane + (int64_t)y * c->W_OUT + x;
        if (c->out_f16) {
            uint16_t* out = (uint16_t*)c->out;
            out[o] = orc_f32_to_f16(R);
            out[o + plane] = orc_f32_to_f16(G);
            out[o + 2 * plane] = orc_f32_to_f16(B);
        } else {
            float* out = (float*)c->out;
            out[o] = R;
            out[o + plane] = G;
            out[o + 2 * plane] = B;
        }
    }
}

int orc_nv12_decode(const uint8_t* nv12, int B, int H_IN, int W_IN, int H_OUT, int W_OUT, int out_f16,
                    void* out, int nthreads)
{
    if (nv12 == NULL || out == NULL) return 1;
    if (B < 0 || H_IN < 2 || W_IN < 2 || H_OUT < 1 || W_OUT < 1) return 2;
    nv12_ctx c;
    c.nv12 = nv12;
    c.H_IN = H_IN;
    c.W_IN = W_IN;
    c.H_OUT = H_OUT;
    c.W_OUT = W_OUT;
    c.out_f16 = out_f16;
    c.out = out;
    /* nv12_decode_kernel.cu:213-216 */
    c.sy_h = (float)H_IN / (float)H_OUT;
    c.sy_w = (float)W_IN / (float)W_OUT;
    c.suv_h = (float)(H_IN >> 1) / (float)H_OUT;
    c.suv_w = (float)(W_IN >> 1) / (float)W_OUT;
    orc_parallel_for((int64_t)B * H_OUT, nthreads, nv12_body, &c);
    return 0;
}

/* ------------------------------------------------------------------ */
/* Disparity regression (no reference counterpart; the formula is the  */
/* specification): disp = sum_d d * softmax_d(s * cost), in double.    */
/* ------------------------------------------------------------------ */

typedef struct {
    const void* cost;
    int in_f16, out_f16;
    int D, H, W;
    double sign;
    void* out;
} disp_ctx;

static void disp_body(void* vctx, int64_t row)
{
    const disp_ctx* c = (const disp_ctx*)vctx;
    const int64_t plane = (int64_t)c->H * c->W;
    const int64_t b = row / c->H, h = row % c->H;
    for (int w = 0; w < c->W; ++w) {
        const int64_t base = b * c->D * plane + h * c->W + w;
        double m = -INFINITY;
        for (int d = 0; d < c->D; ++d) {
            const int64_t i = base + (int64_t)d * plane;
            const double x = c->sign * (c->in_f16 ? (double)orc_f16_to_f32(((const uint16_t*)c->cost)[i])
                                                  : (double)((const float*)c->cost)[i]);
            if (x > m) m = x;
        }
        double s = 0.0, t = 0.0;
        for (int d = 0; d < c->D; ++d) {
            const int64_t i = base + (int64_t)d * plane;
            const double x = c->sign * (c->in_f16 ? (double)orc_f16_to_f32(((const uint16_t*)c->cost)[i])
                                                  : (double)((const float*)c->cost)[i]);
            const double e = exp(x - m);
            s += e;
            t += (double)d * e;
        }
        const double disp = t / s;
        const int64_t o = b * plane + h * c->W + w;
        if (c->out_f16) ((uint16_t*)c->out)[o] = half_from_double(disp);
        else ((float*)c->out)[o] = (float)disp;
    }
}

int orc_disparity_regression(const void* cost, int in_f16, int B, int D, int H, int W, int mode, int out_f16,
                             void* out, int nthreads)
{
    if (cost == NULL || out == NULL) return 1;
    if (B < 0 || D < 1 || H < 0 || W < 0 || (mode != 0 && mode != 1)) return 2;
    disp_ctx c;
    c.cost = cost;
    c.in_f16 = in_f16;
    c.out_f16 = out_f16;
    c.D = D;
    c.H = H;
    c.W = W;
    c.sign = mode == 1 ? -1.0 : 1.0;
    c.out = out;
    orc_parallel_for((int64_t)B * H, nthreads, disp_body, &c);
    return 0;
}

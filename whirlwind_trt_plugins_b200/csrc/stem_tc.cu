// stem_tc.cu -- 3x3x3 Conv3d stem (G -> Cout, pad 1, folded-BN bias, ReLU or
// ReLU6) as an implicit GEMM on the sm_100a tensor cores, optionally fused
// with the group-wise correlation that produces its input volume.
//
//   vol[b, g, d, h, w]  = group-wise correlation of left/right (fused mode), or
//                         read from a [B, G, D, H, W] tensor (volume mode)
//   out[b, o, d, h, w]  = act( sum_{g,kd,kh,kw} W[o,g,kd,kh,kw] * vol[b,g,d+kd-1,h+kh-1,w+kw-1] + bias[o] )
//
// Work decomposition
// ------------------
// A CTA owns one batch item, an 8-column tile [w0, w0+8) of the image and a
// strip of S output rows.  It streams "volume rows" u = h0-1 .. h0+S (one
// image row of the volume: all D disparities x 10 columns incl. halo x all G
// groups) through shared memory:
//
//   producer warps  compute volume row u (fused: the correlation, bit-identical
//                   to the CorrVolume kernels; volume mode: a gather) into a
//                   shared buffer in the UMMA K-major layout
//                       [group octet][d' = d+1][w' = w-w0+1][8 groups x fp16]
//   MMA warp        for each 128-voxel M-block (16 disparities x 8 columns) and
//                   each K-step (two 8-group octets of one or two (kd, kw) taps)
//                   issues one tcgen05.mma with N = 3 * Cout: the three kh taps
//                   are folded into N, so the instruction adds volume row u's
//                   contribution to output rows u+1, u, u-1 at once.  The (kd, kw)
//                   taps are start-address shifts of the same shared buffer.
//   epilogue warps  when output row u-1 is complete, read its accumulators out
//                   of tensor memory, add the bias, apply the activation, store
//                   fp16, and zero the slot for reuse.
//
// Tensor-memory accumulators: per M-block three Cout-column slots; output row
// r lives in slot r mod 3.  The MMA always writes all three slots, so which kh
// lands in which slot rotates with u; the B operand (weights) is stored as five
// Cout-row blocks [kh2, kh1, kh0, kh2, kh1] and the descriptor start selects
// the rotation (rot = (1 - u) mod 3).
//
// Why N = 3*Cout: on B200 an M=128 SS tcgen05.mma costs
// max(N/2, (4096 + 32 N)/128) cycles (shared-memory read bound below N=128;
// measured), so N = Cout = 32 would run at 40 % of peak and N = 96 at ~86 %.
//
// Synchronisation (mbarriers, all waits bounded):
//   vol_full[2]   producers -> MMA        volume buffer ready
//   vol_empty[2]  MMA (commit) -> producers   all MMAs reading it finished
//   acc_full[m]   MMA (commit) -> epilogue    row u-1 of M-block m complete
//   acc_empty[m]  epilogue -> MMA             row u-1's slot drained and zeroed
// A wait that expires records an error code in the device error word and the
// thread stops issuing; the kernel then winds down and frees its TMEM.

#include "umma.cuh"
#include "ww_common.cuh"

#include <algorithm>

namespace ww {

int corr_scale_div_grouped(bool is_half, int B, int C, int G, int H, int W, int D, int sm_count) noexcept;

namespace {

using namespace umma;

constexpr int kWt = 8;             // output columns per tile
constexpr int kWtp = kWt + 2;      // volume columns staged (1-column halo each side)
constexpr int kEpiWarps = 4;       // one per TMEM lane quadrant
constexpr int kMmaWarp = 4;
constexpr int kProdWarp0 = 5;
constexpr int kProdWarps = 8;
constexpr int kProdThreads = kProdWarps * 32;
constexpr int kThreads = (kProdWarp0 + kProdWarps) * 32;  // 416
constexpr int kMaxMB = 10;         // M-blocks per CTA (TMEM: kMaxMB * 3 * 16 <= 512)
constexpr int kLStageW = 24;       // staged left columns [w0-8, w0+16)

struct StemParams {
    const __half* vol;    // volume mode: [B, G, D, H, W]
    const __half* left;   // fused mode:  [B, C, in_rows, W]
    const __half* right;
    const __half* w;      // [Cout, G, 27]
    const __half* bias;   // [Cout]
    __half* out;          // [B, Cout, D, out_rows, W]
    int* err;
    int B, C, G, H, W, D, Cout, act;
    int in_row0, in_rows, out_row0, out_rows;
    int Cg, KG, Dp, n_mb, nsteps, strip, n_strips, n_wtiles;
    int scale_div;
    float inv_cg;
    int vec_ok;
    int rstage_w;             // staged right columns
    uint32_t tmem_cols;
    uint32_t off_b, off_vol, vol_buf_bytes, lbo_vol, off_stage, stage_buf_bytes, off_bar;
};

// K-step s -> (tap, group octet) of its two 8-channel core matrices.
// Steps 0 .. 9*(KG/2)-1 pair octets (2j, 2j+1) of one tap; if KG is odd, the
// last octet of consecutive taps is paired across taps (0,1),(2,3),(4,5),
// (6,7),(8,-), the lone one with a zero-weight partner.
struct StepInfo {
    int t0, kg0, t1, kg1;  // t1 < 0: dummy partner
};

__device__ __forceinline__ StepInfo step_info(int s, int KG)
{
    const int nfull = KG >> 1;
    StepInfo si;
    if (s < 9 * nfull) {
        const int t = s / nfull, j = s - t * nfull;
        si.t0 = t;
        si.kg0 = 2 * j;
        si.t1 = t;
        si.kg1 = 2 * j + 1;
    } else {
        const int q = s - 9 * nfull;
        si.t0 = 2 * q;
        si.kg0 = KG - 1;
        si.t1 = (2 * q + 1 < 9) ? 2 * q + 1 : -1;
        si.kg1 = KG - 1;
    }
    return si;
}

__device__ __forceinline__ uint32_t tap_shift(int t)  // bytes, tap t = kd*3 + kw
{
    const int kd = t / 3, kw = t - 3 * (t / 3);
    return static_cast<uint32_t>((kd * kWtp + kw) * 16);
}

__device__ __forceinline__ float act_apply(float v, int act)
{
    v = fmaxf(v, 0.0f);
    return act ? fminf(v, 6.0f) : v;
}

// Bounded mbarrier wait; on expiry record the error once and return false.
__device__ __forceinline__ bool wait_or_fail(uint32_t bar, uint32_t parity, int* err, int site)
{
    if (mbar_wait(bar, parity)) return true;
    record_device_error(err, kErrMbarTimeout | site);
    return false;
}

template <int COUTP, bool FUSED>
__global__ void __launch_bounds__(kThreads, 1) stem_tc_kernel(const StemParams p)
{
    extern __shared__ __align__(1024) uint8_t smem[];
    constexpr int NR = 5 * COUTP;      // rows of the rotated B image
    constexpr int N = 3 * COUTP;       // MMA N
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // ---- tile coordinates ----
    int t = blockIdx.x;
    const int strip = t % p.n_strips;
    t /= p.n_strips;
    const int wt = t % p.n_wtiles;
    const int b = t / p.n_wtiles;
    const int w0 = wt * kWt;
    const int r0 = p.out_row0 + strip * p.strip;                    // first output row
    const int r1 = min(r0 + p.strip, p.out_row0 + p.out_rows);     // one past last
    const int u_first = r0 - 1;
    const int n_iter = (r1 - r0) + 2;                              // volume rows u_first .. r1
    const int Dtp = p.Dp + 2;

    uint8_t* sB = smem + p.off_b;
    uint8_t* sVol = smem + p.off_vol;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_bar);
    uint64_t* vol_full = bars;           // [2]
    uint64_t* vol_empty = bars + 2;      // [2]
    uint64_t* acc_full = bars + 4;       // [kMaxMB]
    uint64_t* acc_empty = bars + 4 + kMaxMB;
    uint64_t* final_bar = bars + 4 + 2 * kMaxMB;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 5 + 2 * kMaxMB);
    volatile int* prod_abort = reinterpret_cast<volatile int*>(bars + 5 + 2 * kMaxMB) + 1;

    // ---- set-up: barriers, TMEM, B image, zeroed volume buffers ----
    if (threadIdx.x == 0) {
        mbar_init(smem_addr(&vol_full[0]), 1);
        mbar_init(smem_addr(&vol_full[1]), 1);
        mbar_init(smem_addr(&vol_empty[0]), 1);
        mbar_init(smem_addr(&vol_empty[1]), 1);
        for (int m = 0; m < p.n_mb; ++m) {
            mbar_init(smem_addr(&acc_full[m]), 1);
            mbar_init(smem_addr(&acc_empty[m]), kEpiWarps);
        }
        mbar_init(smem_addr(final_bar), 1);
        *prod_abort = 0;
        mbar_fence_init();
    }
    if (warp == kMmaWarp) tmem_alloc(smem_addr(tmem_slot), p.tmem_cols);

    // B image: step s, chunk c, row n (= blk*COUTP + o), 8 fp16 of consecutive groups.
    for (int i = threadIdx.x; i < p.nsteps * 2 * NR; i += kThreads) {
        const int n = i % NR;
        const int sc = i / NR;
        const int c = sc & 1, s = sc >> 1;
        const StepInfo si = step_info(s, p.KG);
        const int tap = c ? si.t1 : si.t0;
        const int kg = c ? si.kg1 : si.kg0;
        const int blk = n / COUTP, o = n - blk * COUTP;
        const int kh = (2 - blk + 3) % 3;
        __align__(16) __half v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int g = kg * 8 + e;
            float x = 0.0f;
            if (tap >= 0 && o < p.Cout && g < p.G) {
                const int kd = tap / 3, kw = tap - 3 * (tap / 3);
                x = __half2float(p.w[(i64(o) * p.G + g) * 27 + kd * 9 + kh * 3 + kw]);
            }
            v[e] = __float2half_rn(x);
        }
        *reinterpret_cast<uint4*>(sB + static_cast<size_t>(i) * 16) = *reinterpret_cast<uint4*>(v);
    }
    // Both volume buffers start as zeros: halo planes and padding stay zero.
    for (uint32_t i = threadIdx.x * 16; i < 2 * p.vol_buf_bytes; i += kThreads * 16)
        *reinterpret_cast<uint4*>(sVol + i) = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem_base = *tmem_slot;

    if (warp < kEpiWarps) {
        // Zero this quadrant's lanes of every accumulator column.
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(warp * 32) << 16);
        const uint32_t zeros[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int c = 0; c < p.n_mb * N; c += 8) tmem_st8(lane_base + c, zeros);
        tmem_wait_st();
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();

    if (warp < kEpiWarps) {
        // ======================= epilogue =======================
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(warp * 32) << 16);
        const int rr = warp * 32 + lane;  // M row
        const int w = w0 + (rr & 7);
        const int dsub = rr >> 3;         // 0..15
        float bias[COUTP];
#pragma unroll
        for (int o = 0; o < COUTP; ++o) bias[o] = (o < p.Cout) ? __half2float(p.bias[o]) : 0.0f;
        const int64_t plane_out = i64(p.out_rows) * p.W;
        bool ok = true;
        for (int it = 0; it < n_iter && ok; ++it) {
            const int r = u_first + it - 1;  // output row completed by this volume row
            const int slot = ((r % 3) + 3) % 3;
            for (int m = 0; m < p.n_mb; ++m) {
                if (!wait_or_fail(smem_addr(&acc_full[m]), it & 1, p.err, 1)) { ok = false; break; }
                fence_after_sync();
                uint32_t acc[COUTP];
                const uint32_t col = lane_base + m * N + slot * COUTP;
#pragma unroll
                for (int c = 0; c < COUTP; c += 16) {
                    uint32_t v16[16];
                    tmem_ld16(col + c, v16);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) acc[c + j] = v16[j];
                }
                const uint32_t zeros[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
                for (int c = 0; c < COUTP; c += 8) tmem_st8(col + c, zeros);
                tmem_wait_st();
                fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_addr(&acc_empty[m]));
                const int d = m * 16 + dsub;
                if (r >= r0 && r < r1 && d < p.D && w < p.W) {
                    __half* op = p.out + ((i64(b) * p.Cout) * p.D + d) * plane_out +
                                 i64(r - p.out_row0) * p.W + w;
                    const int64_t ostride = i64(p.D) * plane_out;
#pragma unroll
                    for (int o = 0; o < COUTP; ++o)
                        if (o < p.Cout)
                            op[o * ostride] = __float2half_rn(act_apply(__uint_as_float(acc[o]) + bias[o], p.act));
                }
            }
        }
    } else if (warp == kMmaWarp) {
        // ======================= MMA issue =======================
        constexpr uint32_t idesc = idesc_f16_f32(128, N);
        bool ok = true;
        for (int it = 0; it < n_iter && ok; ++it) {
            const int u = u_first + it;
            const int vb = it & 1;
            if (lane == 0) ok = wait_or_fail(smem_addr(&vol_full[vb]), (it >> 1) & 1, p.err, 2);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            fence_after_sync();
            const bool active = (u >= 0 && u < p.H);
            const int rot = (((1 - u) % 3) + 3) % 3;
            const uint32_t vol_addr = smem_addr(sVol + vb * p.vol_buf_bytes);
            const uint32_t b_addr = smem_addr(sB) + rot * COUTP * 16;
            for (int m = 0; m < p.n_mb; ++m) {
                if (it > 0) {
                    if (lane == 0) ok = wait_or_fail(smem_addr(&acc_empty[m]), (it - 1) & 1, p.err, 3);
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok) break;
                    fence_after_sync();
                }
                if (lane == 0) {
                    if (active) {
                        const uint32_t a_m = vol_addr + m * 16 * kWtp * 16;
                        const uint32_t d_tmem = tmem_base + m * N;
                        for (int s = 0; s < p.nsteps; ++s) {
                            const StepInfo si = step_info(s, p.KG);
                            const uint32_t off0 = si.kg0 * p.lbo_vol + tap_shift(si.t0);
                            const uint32_t off1 = si.t1 >= 0 ? si.kg1 * p.lbo_vol + tap_shift(si.t1) : off0 + 16;
                            const uint64_t adesc = smem_desc(a_m + off0, off1 - off0, kWtp * 16);
                            const uint64_t bdesc = smem_desc(b_addr + s * 2 * NR * 16, NR * 16, 128);
                            mma_f16_ss(d_tmem, adesc, bdesc, idesc, 1);
                        }
                    }
                    mma_commit(smem_addr(&acc_full[m]));
                }
                __syncwarp();
            }
            if (!ok) break;
            if (lane == 0) mma_commit(smem_addr(&vol_empty[vb]));
            __syncwarp();
        }
    } else {
        // ======================= producers =======================
        const int ptid = threadIdx.x - kProdWarp0 * 32;
        const int Cg = p.Cg;
        __half* stageL = reinterpret_cast<__half*>(smem + p.off_stage);
        __half* stageR = stageL + 8 * Cg * kLStageW;
        const int rbase = w0 - 8 * ((p.D + 7) / 8);  // first staged right column (multiple of 8)
        const int rw = p.rstage_w;
        // All producer threads take the same path through every `bar.sync 1`:
        // a failed wait on thread 0 is broadcast through prod_abort and every
        // producer leaves the loop at the same barrier.
        for (int it = 0; it < n_iter; ++it) {
            const int u = u_first + it;
            const int vb = it & 1;
            if (it >= 2) {
                if (ptid == 0 && !wait_or_fail(smem_addr(&vol_empty[vb]), ((it - 2) >> 1) & 1, p.err, 4))
                    *prod_abort = 1;
                asm volatile("bar.sync 1, %0;\n" ::"r"(kProdThreads) : "memory");
                if (*prod_abort) break;
            }
            if (u >= 0 && u < p.H) {
                uint8_t* vbuf = sVol + vb * p.vol_buf_bytes;
                const int urow = u - p.in_row0;
                for (int kg = 0; kg < p.KG; ++kg) {
                    if (FUSED) {
                        // Stage the octet's 8*Cg channels of left [w0-8, w0+16) and
                        // right [rbase, rbase+rw) of row u (zeros off the image).
                        const int nch = 8 * Cg;
                        const int c0 = kg * 8 * Cg;
                        const int nvl = kLStageW / 8, nvr = rw / 8;
                        for (int i = ptid; i < nch * (nvl + nvr); i += kProdThreads) {
                            const bool isL = i < nch * nvl;
                            const int j = isL ? i : i - nch * nvl;
                            const int nv = isL ? nvl : nvr;
                            const int lc = j / nv, xv = (j - lc * nv) * 8;
                            const int c = c0 + lc;
                            const int x = (isL ? w0 - 8 : rbase) + xv;
                            __half* dst = (isL ? stageL + lc * kLStageW : stageR + lc * rw) + xv;
                            const __half* srow = (isL ? p.left : p.right) +
                                                 ((i64(b) * p.C + c) * p.in_rows + urow) * p.W;
                            if (c < p.C && p.vec_ok && x >= 0 && x + 8 <= p.W) {
                                *reinterpret_cast<uint4*>(dst) = __ldg(reinterpret_cast<const uint4*>(srow + x));
                            } else {
#pragma unroll
                                for (int k = 0; k < 8; ++k) {
                                    const int xx = x + k;
                                    dst[k] = (c < p.C && xx >= 0 && xx < p.W) ? srow[xx] : __float2half_rn(0.0f);
                                }
                            }
                        }
                        asm volatile("bar.sync 1, %0;\n" ::"r"(kProdThreads) : "memory");
                        // Item = (group e of the octet, column pair, 8-disparity run).
                        const int n_pairs = kWtp / 2;
                        const int n_runs = p.Dp / 8;
                        for (int item = ptid; item < 8 * n_pairs * n_runs; item += kProdThreads) {
                            const int e = item % 8;
                            const int rest = item / 8;
                            const int pr = rest % n_pairs;
                            const int run = rest / n_pairs;
                            const int g = kg * 8 + e;
                            float acc[2][8];
#pragma unroll
                            for (int j = 0; j < 2; ++j)
#pragma unroll
                                for (int dd = 0; dd < 8; ++dd) acc[j][dd] = 0.0f;
                            const int wp0 = 2 * pr;                 // w' of the pair
                            const int wabs = w0 - 1 + wp0;          // absolute column of j = 0
                            const int d0 = run * 8;
                            // right index for (j, dd): (wabs + j - (d0 + dd)) - rbase
                            const int rb = wabs - d0 - 7 - rbase;   // index of (j=0, dd=7)
                            if (g < p.G) {
                                for (int cc = 0; cc < Cg; ++cc) {
                                    const int lc = e * Cg + cc;
                                    const __half* lp = stageL + lc * kLStageW + (wabs - (w0 - 8));
                                    const __half* rp = stageR + lc * rw + rb;
                                    float lv[2], rv[9];
                                    lv[0] = __half2float(lp[0]);
                                    lv[1] = __half2float(lp[1]);
#pragma unroll
                                    for (int k = 0; k < 9; ++k) rv[k] = (rb + k >= 0) ? __half2float(rp[k]) : 0.0f;
#pragma unroll
                                    for (int j = 0; j < 2; ++j)
#pragma unroll
                                        for (int dd = 0; dd < 8; ++dd)
                                            acc[j][dd] = __fmaf_rn(lv[j], rv[7 - dd + j], acc[j][dd]);
                                }
                            }
                            const float cgf = static_cast<float>(Cg);
#pragma unroll
                            for (int j = 0; j < 2; ++j) {
                                const int wa = wabs + j;
#pragma unroll
                                for (int dd = 0; dd < 8; ++dd) {
                                    const int d = d0 + dd;
                                    float v = 0.0f;
                                    if (g < p.G && wa >= 0 && wa < p.W && d < p.D && wa - d >= 0)
                                        v = p.scale_div ? __fdiv_rn(acc[j][dd], cgf) : __fmul_rn(acc[j][dd], p.inv_cg);
                                    const int dp = d + 1;
                                    if (dp < Dtp) {
                                        __half* dst = reinterpret_cast<__half*>(
                                            vbuf + kg * p.lbo_vol + (dp * kWtp + wp0 + j) * 16) + e;
                                        *dst = __float2half_rn(v);
                                    }
                                }
                            }
                        }
                        asm volatile("bar.sync 1, %0;\n" ::"r"(kProdThreads) : "memory");
                    } else {
                        // Volume mode: gather vol[b, g, d, u, w] into the octet's rows.
                        const int64_t plane = i64(p.H) * p.W;
                        for (int i = ptid; i < 8 * p.D * kWtp; i += kProdThreads) {
                            const int e = i % 8;
                            const int rest = i / 8;
                            const int wp = rest % kWtp;
                            const int d = rest / kWtp;
                            const int g = kg * 8 + e;
                            const int wa = w0 - 1 + wp;
                            __half v = __float2half_rn(0.0f);
                            if (g < p.G && wa >= 0 && wa < p.W)
                                v = p.vol[((i64(b) * p.G + g) * p.D + d) * plane + i64(u) * p.W + wa];
                            *(reinterpret_cast<__half*>(vbuf + kg * p.lbo_vol + ((d + 1) * kWtp + wp) * 16) + e) = v;
                        }
                    }
                }
            }
            fence_proxy_async_smem();
            asm volatile("bar.sync 1, %0;\n" ::"r"(kProdThreads) : "memory");
            if (ptid == 0) mbar_arrive(smem_addr(&vol_full[vb]));
        }
    }

    // ---- teardown ----
    // Every MMA this CTA issued has completed before TMEM is released (on the
    // normal path this is already implied by the last acc_full wait; after a
    // timed-out wait it is not).
    if (warp == kMmaWarp) {
        if (lane == 0) {
            mma_commit(smem_addr(final_bar));
            wait_or_fail(smem_addr(final_bar), 0, p.err, 5);
        }
        __syncwarp();
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (warp == kMmaWarp) tmem_dealloc(tmem_base, p.tmem_cols);
}

uint32_t pow2_cols(uint32_t c)
{
    uint32_t r = 32;
    while (r < c) r <<= 1;
    return r;
}

}  // namespace

int stem_tc_launch(const void* vol, const void* left, const void* right, const void* w, const void* b,
                   void* out, int B, int C, int G, int H, int W, int D, int Cout, int act, int in_row0,
                   int in_rows, int out_row0, int out_rows, cudaStream_t stream) noexcept
{
    const bool fused = (vol == nullptr);
    if (w == nullptr || b == nullptr || out == nullptr) return WW_ERR_NULL_POINTER;
    if (B < 0 || C <= 0 || G <= 0 || H < 0 || W < 0 || D < 0 || Cout <= 0) return WW_ERR_INVALID_SHAPE;
    if (fused && C % G != 0) return WW_ERR_INVALID_SHAPE;
    if (act != WW_ACT_RELU && act != WW_ACT_RELU6) return WW_ERR_INVALID_SHAPE;
    if (out_rows < 0 || out_row0 < 0 || out_row0 + out_rows > H) return WW_ERR_INVALID_SHAPE;
    if (in_rows < 0 || in_row0 < 0 || in_row0 + in_rows > H) return WW_ERR_INVALID_SHAPE;
    if (out_rows > 0) {
        // the input band must hold rows [out_row0-1, out_row0+out_rows+1) clipped to [0,H)
        const int need0 = out_row0 > 0 ? out_row0 - 1 : 0;
        const int need1 = out_row0 + out_rows < H ? out_row0 + out_rows + 1 : H;
        if (in_row0 > need0 || in_row0 + in_rows < need1) return WW_ERR_INVALID_SHAPE;
    }
    if (B == 0 || W == 0 || D == 0 || out_rows == 0) return WW_SUCCESS;
    if (Cout > 32) return WW_ERR_UNSUPPORTED;

    DeviceInfo dev;
    if (current_device_info(&dev) != WW_SUCCESS || dev.cc_major < 10) return WW_ERR_DEVICE;

    const int coutp = Cout <= 16 ? 16 : 32;
    const int KG = (G + 7) / 8;
    const int Dp = (D + 15) / 16 * 16;
    const int n_mb = Dp / 16;
    if (n_mb * 3 * coutp > 512 || n_mb > kMaxMB) return WW_ERR_UNSUPPORTED;
    const int nsteps = 9 * (KG / 2) + ((KG & 1) ? 5 : 0);
    const int Cg = fused ? C / G : 1;

    StemParams p{};
    p.vol = static_cast<const __half*>(vol);
    p.left = static_cast<const __half*>(left);
    p.right = static_cast<const __half*>(right);
    p.w = static_cast<const __half*>(w);
    p.bias = static_cast<const __half*>(b);
    p.out = static_cast<__half*>(out);
    p.err = device_error_slot();
    if (p.err == nullptr) return WW_ERR_DEVICE;
    p.B = B; p.C = C; p.G = G; p.H = H; p.W = W; p.D = D; p.Cout = Cout; p.act = act;
    p.in_row0 = in_row0; p.in_rows = in_rows; p.out_row0 = out_row0; p.out_rows = out_rows;
    p.Cg = Cg; p.KG = KG; p.Dp = Dp; p.n_mb = n_mb; p.nsteps = nsteps;
    p.n_wtiles = (W + kWt - 1) / kWt;
    p.scale_div = fused ? corr_scale_div_grouped(true, B, C, G, H, W, D, dev.sm_count) : 0;
    p.inv_cg = 1.0f / static_cast<float>(Cg);
    p.vec_ok = (W % 8 == 0) && (reinterpret_cast<uintptr_t>(left) % 16 == 0) &&
               (reinterpret_cast<uintptr_t>(right) % 16 == 0);
    p.rstage_w = 16 + 8 * ((D + 7) / 8);
    p.tmem_cols = pow2_cols(static_cast<uint32_t>(n_mb * 3 * coutp));

    // shared-memory layout
    uint32_t off = 0;
    p.off_b = off;
    off += static_cast<uint32_t>(nsteps) * 2 * 5 * coutp * 16;
    off = (off + 127) & ~127u;
    p.off_vol = off;
    p.lbo_vol = static_cast<uint32_t>((Dp + 2) * kWtp * 16);
    // + a zeroed 128-byte guard: the zero-weight partner of a lone octet
    // (step_info, t1 < 0) reads one 16-byte position past the last plane.
    p.vol_buf_bytes = p.lbo_vol * KG + 128;
    off += 2 * p.vol_buf_bytes;
    off = (off + 127) & ~127u;
    p.off_stage = off;
    p.stage_buf_bytes = fused ? static_cast<uint32_t>(8 * Cg * (kLStageW + p.rstage_w) * 2) : 0;
    off += p.stage_buf_bytes;
    off = (off + 127) & ~127u;
    p.off_bar = off;
    off += (5 + 2 * kMaxMB) * 8 + 16;
    const size_t smem = off;
    if (smem > static_cast<size_t>(dev.smem_optin)) return WW_ERR_UNSUPPORTED;

    // Strip length: minimise (waves of CTAs) x (rows streamed per CTA).
    const long long col_tiles = static_cast<long long>(B) * p.n_wtiles;
    const int ctas_per_sm = static_cast<int>(std::max<size_t>(1, std::min<size_t>(
        dev.smem_optin / (smem + 1024), 512 / p.tmem_cols)));
    const long long slots = static_cast<long long>(dev.sm_count) * ctas_per_sm;
    int best_s = out_rows;
    long long best_cost = -1;
    for (int s = 1; s <= out_rows; ++s) {
        const long long tiles = col_tiles * ((out_rows + s - 1) / s);
        const long long waves = (tiles + slots - 1) / slots;
        const long long cost = waves * (s + 2);
        if (best_cost < 0 || cost < best_cost) { best_cost = cost; best_s = s; }
    }
    p.strip = best_s;
    p.n_strips = (out_rows + best_s - 1) / best_s;
    const long long grid = col_tiles * p.n_strips;
    if (grid > 0x7fffffffLL) return WW_ERR_UNSUPPORTED;

    auto launch = [&](auto kernel) -> int {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
            cudaSuccess)
            return launch_status("ww_cost_stem3d");
        kernel<<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(p);
        return launch_status(fused ? "ww_corr_cost_stem3d" : "ww_cost_stem3d");
    };
    if (coutp == 16) return fused ? launch(stem_tc_kernel<16, true>) : launch(stem_tc_kernel<16, false>);
    return fused ? launch(stem_tc_kernel<32, true>) : launch(stem_tc_kernel<32, false>);
}

}  // namespace ww

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
// groups) through shared memory.  Warp roles:
//
//   loader (1 warp)     stages, per group octet ("job"), the left columns
//                       [w0-8, w0+16) and right columns [w0-8*ceil(D/8), w0+16)
//                       of the octet's channels into a two-slot ring with one
//                       1-D bulk copy (TMA engine) per channel row and side;
//                       completion is counted in bytes on an mbarrier.
//   producers (8 warps) compute the octet's correlation (fused; bit-identical
//                       to the CorrVolume kernels) or gather it (volume mode)
//                       into the volume buffer in the UMMA K-major layout
//                           [group octet][d' = d+1][w' = w-w0+1][8 groups x fp16]
//   MMA (1 warp)        for each 128-voxel M-block (16 disparities x 8 columns)
//                       and K-step (two 8-group octets of one or two (kd, kw)
//                       taps) issues one tcgen05.mma with N = 3 * Cout: the three
//                       kh taps are folded into N, so one instruction adds volume
//                       row u's contribution to output rows u+1, u, u-1.  The
//                       (kd, kw) taps are start-address shifts of the same buffer.
//   epilogue (4 warps)  when output row u-1 is complete, read its accumulators
//                       out of tensor memory, add the bias, apply the
//                       activation, store fp16, and zero the slot for reuse.
//
// Tensor-memory accumulators: per M-block three Cout-column slots; output row
// r lives in slot r mod 3.  The MMA always writes all three slots, so which kh
// lands in which slot rotates with u; the B operand (weights) is stored as five
// Cout-row blocks [kh2, kh1, kh0, kh2, kh1] and the descriptor start selects
// the rotation (rot = (1 - u) mod 3).
//
// Measured facts that shape this (B200): an M=128 SS tcgen05.mma costs
// max(N/2, (4096 + 32 N)/128) cycles (shared-memory read bound below N=128),
// so N = 3*Cout = 96 runs at ~86 % of peak where N = Cout would run at 40 %;
// MMAs accumulating into the same columns back to back cost ~93 cycles each,
// so the MMA warp interleaves two accumulator chains; descriptors come from
// kernel parameters (constant bank, uniform registers), never from shared
// memory, so the issue path does not queue behind the producers' loads.
//
// Synchronisation (mbarriers, every wait bounded):
//   stage_full[2]   loader (bulk-copy bytes) -> producers
//   stage_empty[2]  producers -> loader
//   vol_full[2]     producers -> MMA        volume buffer ready
//   vol_empty[2]    MMA (commit) -> producers   all MMAs reading it finished
//   acc_full[m]     MMA (commit) -> epilogue    row u-1 of M-block m complete
//   acc_empty[m]    epilogue -> MMA             row u-1's slot drained and zeroed
// A wait that expires records an error code in the device error word; the
// waiting role stops, the others run into their own bounded waits, and the
// CTA winds down and frees its tensor memory.

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
constexpr int kLoadWarp = 5;
constexpr int kProdWarp0 = 6;
constexpr int kProdWarps = 8;
constexpr int kThreads = (kProdWarp0 + kProdWarps) * 32;  // 448
constexpr int kMaxMB = 10;         // M-blocks per CTA (TMEM: kMaxMB * 3 * 16 <= 512)
constexpr int kLStageW = 24;       // staged left columns [w0-8, w0+16)
constexpr int kMaxSteps = 32;      // K-steps per M-block (group octets <= 7)
constexpr int kMaxSlots = 4;       // staging ring depth

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
    int n_slots;              // staging ring depth (2..kMaxSlots)
    uint32_t tmem_cols;
    uint32_t off_b, off_vol, vol_buf_bytes, lbo_vol, off_stage, stage_slot_bytes, stage_group_bytes, off_bar;
    // Per K-step descriptor templates with a zero base address: A relative to a
    // volume buffer, B relative to the B image.  Read with uniform loads.
    uint64_t tmplA[kMaxSteps];
    uint64_t tmplB[kMaxSteps];
};

// K-step s -> (tap, group octet) of its two 8-channel core matrices.
// Steps 0 .. 9*(KG/2)-1 pair octets (2j, 2j+1) of one tap; if KG is odd, the
// last octet of consecutive taps is paired across taps (0,1),(2,3),(4,5),
// (6,7),(8,-), the lone one with a zero-weight partner.
struct StepInfo {
    int t0, kg0, t1, kg1;  // t1 < 0: zero-weight partner
};

__host__ __device__ inline StepInfo step_info(int s, int KG)
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

__host__ __device__ inline uint32_t tap_shift(int t)  // bytes, tap t = kd*3 + kw
{
    const int kd = t / 3, kw = t - 3 * (t / 3);
    return static_cast<uint32_t>((kd * kWtp + kw) * 16);
}

// Host copy of the shared-memory descriptor encoding in umma.cuh (smem_desc).
inline uint64_t host_smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo)
{
    return (static_cast<uint64_t>((saddr >> 4) & 0x3FFFu)) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (static_cast<uint64_t>(1u) << 46);
}

__device__ __forceinline__ float act_apply(float v, int act)
{
    v = fmaxf(v, 0.0f);
    return act ? fminf(v, 6.0f) : v;
}

__device__ __forceinline__ bool elect_one()
{
    uint32_t pred = 0;
    asm volatile("{\n\t.reg .pred P;\n\telect.sync _|P, 0xffffffff;\n\tselp.b32 %0, 1, 0, P;\n\t}\n" : "=r"(pred));
    return pred != 0;
}

// Bounded mbarrier wait; on expiry record the error once and return false.
__device__ __forceinline__ bool wait_or_fail(uint32_t bar, uint32_t parity, int* err, int site)
{
    if (mbar_wait(bar, parity)) return true;
    record_device_error(err, kErrMbarTimeout | site);
    return false;
}

// Whole-warp bounded wait: every lane polls; the warp agrees on the outcome.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, int* err, int site)
{
    const bool ok = wait_or_fail(bar, parity, err, site);
    return __all_sync(0xffffffffu, ok);
}

// Correlation of one group for a 2-column x 8-disparity tile:
//   acc[h][dd] = sum_c L[c][x0 + h] * R[c][x0 + h - dd]   (staged coordinates)
// as one fp32 fma chain per output in channel order (bit-identical to the
// reference).  lp -> L[0][x0] (left rows of kLStageW), rp -> R[0][x0 - 7]
// (right rows of rw, 4-byte aligned).  CG > 0: compile-time channel count,
// fully unrolled so every load is issued ahead of its FMAs; CG == 0: runtime.
template <int CG>
__device__ __forceinline__ void corr_tile(const unsigned short* __restrict__ lp, const __half* __restrict__ rp,
                                          int rw, int cg_rt, float (&acc)[2][8])
{
    const int cg = CG > 0 ? CG : cg_rt;
#pragma unroll
    for (int cc = 0; cc < cg; ++cc) {
        const unsigned short l0 = lp[cc * kLStageW];
        const unsigned short l1 = lp[cc * kLStageW + 1];
        const uint32_t* rq = reinterpret_cast<const uint32_t*>(rp + cc * rw);
        unsigned short r[10];
#pragma unroll
        for (int q = 0; q < 5; ++q) {
            const uint32_t x = rq[q];
            r[2 * q] = static_cast<unsigned short>(x & 0xffffu);
            r[2 * q + 1] = static_cast<unsigned short>(x >> 16);
        }
#pragma unroll
        for (int dd = 0; dd < 8; ++dd) {
            acc[0][dd] = fma_f16f16f32(l0, r[7 - dd], acc[0][dd]);
            acc[1][dd] = fma_f16f16f32(l1, r[8 - dd], acc[1][dd]);
        }
    }
}

template <int COUTP, bool FUSED>
__global__ void __launch_bounds__(kThreads, 1) stem_tc_kernel(const __grid_constant__ StemParams p)
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
    // volume rows inside the image (a contiguous range) and the staging jobs over them
    const int uv0 = max(u_first, 0);
    const int uv1 = min(u_first + n_iter, p.H);
    const int total_jobs = FUSED ? max(0, uv1 - uv0) * p.KG : 0;

    uint8_t* sB = smem + p.off_b;
    uint8_t* sVol = smem + p.off_vol;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_bar);
    uint64_t* vol_full = bars;             // [2]
    uint64_t* vol_empty = bars + 2;        // [2]
    uint64_t* final_bar = bars + 4;
    uint64_t* stage_full = bars + 5;                  // [n_slots]
    uint64_t* stage_empty = stage_full + p.n_slots;   // [n_slots]
    uint64_t* acc_full = stage_empty + p.n_slots;     // [n_mb]
    uint64_t* acc_empty = acc_full + p.n_mb;          // [n_mb]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + p.n_mb);

    // ---- set-up: barriers, TMEM, B image, zeroed volume buffers ----
    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_addr(&vol_full[i]), kProdWarps);
            mbar_init(smem_addr(&vol_empty[i]), 1);
        }
        for (int i = 0; i < p.n_slots; ++i) {
            mbar_init(smem_addr(&stage_full[i]), 32);
            mbar_init(smem_addr(&stage_empty[i]), kProdWarps);
        }
        mbar_init(smem_addr(final_bar), 1);
        for (int m = 0; m < p.n_mb; ++m) {
            mbar_init(smem_addr(&acc_full[m]), 1);
            mbar_init(smem_addr(&acc_empty[m]), kEpiWarps);
        }
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
        const int64_t ostride = i64(p.D) * plane_out;
        bool ok = true;
        for (int it = 0; it < n_iter && ok; ++it) {
            const int r = u_first + it - 1;  // output row completed by this volume row
            const int slot = ((r % 3) + 3) % 3;
            for (int m = 0; m < p.n_mb; ++m) {
                if (!warp_wait(smem_addr(&acc_full[m]), it & 1, p.err, 1)) { ok = false; break; }
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
                    __half* op = p.out + ((i64(b) * p.Cout) * p.D + d) * plane_out + i64(r - p.out_row0) * p.W + w;
#pragma unroll
                    for (int o = 0; o < COUTP; ++o)
                        if (o < p.Cout)
                            op[o * ostride] = __float2half_rn(act_apply(__uint_as_float(acc[o]) + bias[o], p.act));
                }
            }
        }
    } else if (warp == kMmaWarp) {
        // ======================= MMA issue =======================
        // A "chain" is one (volume row, M-block): nsteps MMAs accumulating into
        // the same tensor-memory columns.  Back to back, such a chain runs at
        // ~93 cycles per MMA instead of the ~56 an independent MMA costs, so
        // chains are issued staggered: the second half of chain k-1
        // interleaved with the first half of chain k.  Chain k needs only what
        // chain k-1's predecessors released (its volume row; the drain of its
        // slot two rows back), so there is no bubble at M-block or row
        // boundaries.  The whole warp runs the (uniform) schedule; one elected
        // lane issues.
        constexpr uint32_t idesc = idesc_f16_f32(128, N);
        const int S = p.nsteps;
        const int S1 = (S + 1) / 2;
        const int n_chains = n_iter * p.n_mb;
        const bool stagger = p.n_mb > 1;  // one M-block: chain k waits on chain k-1's drain
        const uint64_t vol_base = smem_addr(sVol) >> 4;
        const uint64_t b_base = smem_addr(sB) >> 4;
        bool ok = true;
        bool prev_live = false, prev_active = false;
        int prev_m = 0, prev_it = 0;
        uint64_t prev_a = 0, prev_b = 0;
        uint32_t prev_d = 0;
        auto issue_range = [&](bool active, uint64_t a_add, uint64_t b_add, uint32_t d, int s0, int s1) {
            if (!active) return;
            for (int st = s0; st < s1; ++st) {
                const uint64_t ad = p.tmplA[st] + a_add, bd = p.tmplB[st] + b_add;
                if (elect_one()) mma_f16_ss(d, ad, bd, idesc, 1);
                __syncwarp();
            }
        };
        auto retire_prev = [&]() {  // second half issued: signal its consumers
            if (elect_one()) {
                mma_commit(smem_addr(&acc_full[prev_m]));
                if (prev_m == p.n_mb - 1) mma_commit(smem_addr(&vol_empty[prev_it & 1]));
            }
            __syncwarp();
            prev_live = false;
        };
        for (int k = 0; k < n_chains && ok; ++k) {
            const int it = k / p.n_mb, m = k - it * p.n_mb;
            const int u = u_first + it;
            if (m == 0) {
                const uint32_t bar = smem_addr(&vol_full[it & 1]);
                if (prev_live && !__all_sync(0xffffffffu, mbar_try_wait(bar, (it >> 1) & 1))) {
                    // the next row is not produced yet: finish the previous chain alone
                    issue_range(prev_active, prev_a, prev_b, prev_d, S1, S);
                    retire_prev();
                }
                if (!warp_wait(bar, (it >> 1) & 1, p.err, 2)) { ok = false; break; }
            }
            if (!stagger && prev_live) {
                issue_range(prev_active, prev_a, prev_b, prev_d, S1, S);
                retire_prev();
            }
            if (it > 0 && !warp_wait(smem_addr(&acc_empty[m]), (it - 1) & 1, p.err, 3)) { ok = false; break; }
            fence_after_sync();
            const bool active = (u >= 0 && u < p.H);
            const int rot = (((1 - u) % 3) + 3) % 3;
            const uint64_t b_add = b_base + static_cast<uint64_t>((rot * COUTP * 16) >> 4);
            const uint64_t a_add = vol_base + static_cast<uint64_t>(((it & 1) * p.vol_buf_bytes + m * 16 * kWtp * 16) >> 4);
            const uint32_t d = tmem_base + m * N;
            if (prev_live) {
                // interleave: previous chain steps [S1, S) with this chain's [0, S1)
                for (int j = 0; j < S1; ++j) {
                    const bool do_prev = prev_active && S1 + j < S;
                    const uint64_t pa = p.tmplA[S1 + j < S ? S1 + j : 0] + prev_a;
                    const uint64_t pb = p.tmplB[S1 + j < S ? S1 + j : 0] + prev_b;
                    const uint64_t ca = p.tmplA[j] + a_add, cb = p.tmplB[j] + b_add;
                    if (elect_one()) {
                        if (do_prev) mma_f16_ss(prev_d, pa, pb, idesc, 1);
                        if (active) mma_f16_ss(d, ca, cb, idesc, 1);
                    }
                    __syncwarp();
                }
                retire_prev();
            } else {
                issue_range(active, a_add, b_add, d, 0, S1);
            }
            prev_live = true;
            prev_active = active;
            prev_m = m;
            prev_it = it;
            prev_a = a_add;
            prev_b = b_add;
            prev_d = d;
        }
        if (ok && prev_live) {
            issue_range(prev_active, prev_a, prev_b, prev_d, S1, S);
            retire_prev();
        }
    } else if (warp == kLoadWarp) {
        // ======================= loader =======================
        // Job j = (volume row uv0 + j / KG, group octet j % KG) -> slot j % NS.
        // Per group: left [Cg][24] then right [Cg][rstage_w] fp16, regions
        // padded so consecutive groups start 16 bytes apart modulo 128.  Lanes
        // take whole channel rows and cp.async them in 16-byte vectors (zero
        // fill outside the image); each lane's copies complete onto stage_full.
        if (FUSED) {
            const int Cg = p.Cg;
            const int rw = p.rstage_w;
            const int NS = p.n_slots;
            const int n_runs = (p.D + 7) / 8;
            const int rbase = w0 - 8 * n_runs;
            const int nvr = rw / 8;
            int issued = 0;
            for (int j = 0; j < total_jobs; ++j) {
                const int slot = j % NS;
                if (j >= NS && !warp_wait(smem_addr(&stage_empty[slot]), ((j / NS) - 1) & 1, p.err, 6)) break;
                issued = j + 1;
                uint8_t* sbase = smem + p.off_stage + slot * p.stage_slot_bytes;
                const int urow = uv0 + j / p.KG - p.in_row0;
                const int kg = j % p.KG;
                for (int lc = lane; lc < 8 * Cg; lc += 32) {
                    const int ge = lc / Cg, cc = lc - ge * Cg;
                    const int g = kg * 8 + ge;
                    const bool gv = g < p.G;
                    const int64_t roff = ((i64(b) * p.C + (gv ? g * Cg + cc : 0)) * p.in_rows + urow) * p.W;
                    uint8_t* gdst = sbase + ge * p.stage_group_bytes;
                    for (int v = 0; v < 3 + nvr; ++v) {
                        const bool isL = v < 3;
                        const int x = isL ? (w0 - 8 + 8 * v) : (rbase + 8 * (v - 3));
                        uint8_t* dst = gdst + (isL ? cc * (kLStageW * 2) + 16 * v
                                                   : Cg * (kLStageW * 2) + cc * rw * 2 + 16 * (v - 3));
                        const __half* srow = (isL ? p.left : p.right) + roff;
                        if (p.vec_ok) {
                            const bool in = gv && x >= 0 && x < p.W;  // whole vector (W % 8 == 0)
                            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n"
                                         :
                                         : "r"(smem_addr(dst)), "l"(in ? srow + x : srow), "r"(in ? 16 : 0)
                                         : "memory");
                        } else {
                            __half* d16 = reinterpret_cast<__half*>(dst);
#pragma unroll
                            for (int q = 0; q < 8; ++q) {
                                const int xx = x + q;
                                d16[q] = (gv && xx >= 0 && xx < p.W) ? srow[xx] : __float2half_rn(0.0f);
                            }
                        }
                    }
                }
                if (p.vec_ok) {
                    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n"
                                 :
                                 : "r"(smem_addr(&stage_full[slot]))
                                 : "memory");
                } else {
                    __threadfence_block();
                    mbar_arrive(smem_addr(&stage_full[slot]));
                }
            }
            // Nothing may still be landing in shared memory when the CTA exits.
            asm volatile("cp.async.wait_all;\n" ::: "memory");
            (void)issued;
        }
    } else {
        // ======================= producers =======================
        // Fused mode: lane (e = lane/4, pp = lane%4) of a producer warp computes
        // group e's correlation for a 2-column x 8-disparity tile of the job's
        // octet; stmatrix.trans then writes the eight groups of each position
        // as one 16-byte row of the volume buffer.  Warps run independently,
        // synchronised only through the stage and volume mbarriers.
        const int pw = warp - kProdWarp0;
        const int e = lane >> 2;
        const int pp = lane & 3;
        const int Cg = p.Cg;
        const int rw = p.rstage_w;
        const int n_runs = (p.D + 7) / 8;
        const int n_tasks = n_runs + (n_runs + 3) / 4;
        const float cgf = static_cast<float>(Cg);
        int job = 0;
        bool ok = true;
        for (int it = 0; it < n_iter && ok; ++it) {
            const int u = u_first + it;
            const int vb = it & 1;
            if (it >= 2 && !warp_wait(smem_addr(&vol_empty[vb]), ((it - 2) >> 1) & 1, p.err, 4)) break;
            if (u >= 0 && u < p.H) {
                uint8_t* vbuf = sVol + vb * p.vol_buf_bytes;
                for (int kg = 0; kg < p.KG; ++kg) {
                    if (FUSED) {
                        const int slot = job % p.n_slots;
                        if (!warp_wait(smem_addr(&stage_full[slot]), (job / p.n_slots) & 1, p.err, 7)) { ok = false; break; }
                        const uint8_t* gbase = smem + p.off_stage + slot * p.stage_slot_bytes + e * p.stage_group_bytes;
                        const unsigned short* Ls = reinterpret_cast<const unsigned short*>(gbase);
                        const __half* Rs = reinterpret_cast<const __half*>(gbase + Cg * (kLStageW * 2));
                        const uint32_t vsa = smem_addr(vbuf + kg * p.lbo_vol);
                        const int g = kg * 8 + e;
                        for (int task = pw; task < n_tasks; task += kProdWarps) {
                            const bool nice = task < n_runs;          // columns 0..7, one disparity run
                            const int pr = nice ? pp : 4;              // column pair
                            const int run = nice ? task : 4 * (task - n_runs) + pp;
                            const bool active = run < n_runs && g < p.G;
                            float acc[2][8];
#pragma unroll
                            for (int h = 0; h < 2; ++h)
#pragma unroll
                                for (int dd = 0; dd < 8; ++dd) acc[h][dd] = 0.0f;
                            if (active) {
                                const unsigned short* lp = Ls + 2 * pr + 7;
                                const __half* rp = Rs + 2 * pr - 8 * run - 8 + 8 * n_runs;
                                switch (Cg) {  // fully unrolled for the common group widths
                                    case 4: corr_tile<4>(lp, rp, rw, Cg, acc); break;
                                    case 8: corr_tile<8>(lp, rp, rw, Cg, acc); break;
                                    case 12: corr_tile<12>(lp, rp, rw, Cg, acc); break;
                                    case 16: corr_tile<16>(lp, rp, rw, Cg, acc); break;
                                    default: corr_tile<0>(lp, rp, rw, Cg, acc); break;
                                }
                            }
                            // fp16 values, packed (h = 0 low, h = 1 high) per disparity
                            uint32_t packed[8];
                            const int wa0 = w0 - 1 + 2 * pr;
                            const bool interior = active && wa0 >= 0 && wa0 + 1 < p.W && 8 * run + 7 < p.D &&
                                                  wa0 - (8 * run + 7) >= 0;
                            if (interior && !p.scale_div) {
#pragma unroll
                                for (int dd = 0; dd < 8; ++dd) {
                                    const __half2 h2 = __floats2half2_rn(__fmul_rn(acc[0][dd], p.inv_cg),
                                                                         __fmul_rn(acc[1][dd], p.inv_cg));
                                    packed[dd] = *reinterpret_cast<const uint32_t*>(&h2);
                                }
                            } else {
#pragma unroll
                                for (int dd = 0; dd < 8; ++dd) {
                                    const int d = 8 * run + dd;
                                    uint32_t hv[2];
#pragma unroll
                                    for (int h = 0; h < 2; ++h) {
                                        const int wa = wa0 + h;
                                        float v = 0.0f;
                                        if (active && wa >= 0 && wa < p.W && d < p.D && wa - d >= 0)
                                            v = p.scale_div ? __fdiv_rn(acc[h][dd], cgf) : __fmul_rn(acc[h][dd], p.inv_cg);
                                        hv[h] = __half_as_ushort(__float2half_rn(v));
                                    }
                                    packed[dd] = hv[0] | (hv[1] << 16);
                                }
                            }
                            // Row address this lane supplies: matrix mi = lane/8, row rr = lane%8
                            // -> position of lane-group pp' = rr/2, column h = rr%2, disparity 4s+mi.
                            const int mi = lane >> 3, rr = lane & 7;
                            const int pq = rr >> 1, hq = rr & 1;
                            const int prq = nice ? pq : 4;
                            const int runq = nice ? task : 4 * (task - n_runs) + pq;
#pragma unroll
                            for (int sg = 0; sg < 2; ++sg) {
                                const int dq = 8 * runq + 4 * sg + mi;
                                int pos;
                                if (runq < n_runs) pos = (dq + 1) * kWtp + 2 * prq + hq;
                                else pos = (Dtp - 1) * kWtp + hq;  // inactive: an always-zero plane, zeros written
                                asm volatile(
                                    "stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1, %2, %3, %4};\n"
                                    :
                                    : "r"(vsa + pos * 16), "r"(packed[4 * sg + 0]), "r"(packed[4 * sg + 1]),
                                      "r"(packed[4 * sg + 2]), "r"(packed[4 * sg + 3])
                                    : "memory");
                            }
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(smem_addr(&stage_empty[slot]));
                        ++job;
                    } else {
                        // Volume mode: gather vol[b, g, d, u, w] into the octet's rows.
                        const int64_t plane = i64(p.H) * p.W;
                        for (int i = pw * 32 + lane; i < 8 * p.D * kWtp; i += kProdWarps * 32) {
                            const int ge = i % 8;
                            const int rest = i / 8;
                            const int wp = rest % kWtp;
                            const int d = rest / kWtp;
                            const int g = kg * 8 + ge;
                            const int wa = w0 - 1 + wp;
                            __half v = __float2half_rn(0.0f);
                            if (g < p.G && wa >= 0 && wa < p.W)
                                v = p.vol[((i64(b) * p.G + g) * p.D + d) * plane + i64(u) * p.W + wa];
                            *(reinterpret_cast<__half*>(vbuf + kg * p.lbo_vol + ((d + 1) * kWtp + wp) * 16) + ge) = v;
                        }
                    }
                }
            }
            if (!ok) break;
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_addr(&vol_full[vb]));
        }
    }

    // ---- teardown ----
    // Every MMA this CTA issued has completed before TMEM is released (on the
    // normal path this is already implied by the last acc_full wait; after a
    // timed-out wait it is not).
    if (warp == kMmaWarp) {
        if (elect_one()) {
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
    if (nsteps > kMaxSteps) return WW_ERR_UNSUPPORTED;
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
    p.rstage_w = 16 + 8 * ((D + 7) / 8);  // right columns [w0 - 8*ceil(D/8), w0 + 16)
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
    // Per group: left [Cg][24] then right [Cg][rstage_w] fp16, padded so that
    // consecutive groups start 16 bytes apart modulo 128 (different banks).
    p.stage_group_bytes = static_cast<uint32_t>(((Cg * (kLStageW + p.rstage_w) * 2 + 127) / 128) * 128 + 16);
    p.stage_slot_bytes = fused ? ((8 * p.stage_group_bytes + 127) / 128) * 128 : 0;
    auto bar_bytes = [&](int ns) { return static_cast<uint32_t>((5 + 2 * ns + 2 * n_mb) * 8 + 16); };
    // as many staging slots (2..kMaxSlots) as shared memory holds
    p.n_slots = 2;
    while (p.n_slots < kMaxSlots && off + (p.n_slots + 1) * p.stage_slot_bytes + bar_bytes(p.n_slots + 1) <=
                                        static_cast<uint32_t>(dev.smem_optin))
        ++p.n_slots;
    off += p.n_slots * p.stage_slot_bytes;
    off = (off + 127) & ~127u;
    p.off_bar = off;
    off += bar_bytes(p.n_slots);
    const size_t smem = off;
    if (smem > static_cast<size_t>(dev.smem_optin)) return WW_ERR_UNSUPPORTED;

    // Descriptor templates (base address 0; the kernel adds its buffer bases).
    for (int s = 0; s < nsteps; ++s) {
        const StepInfo si = step_info(s, KG);
        const uint32_t off0 = si.kg0 * p.lbo_vol + tap_shift(si.t0);
        const uint32_t off1 = si.t1 >= 0 ? si.kg1 * p.lbo_vol + tap_shift(si.t1) : off0 + 16;
        p.tmplA[s] = host_smem_desc(off0, off1 - off0, kWtp * 16);
        p.tmplB[s] = host_smem_desc(static_cast<uint32_t>(s * 2 * 5 * coutp * 16), 5 * coutp * 16, 128);
    }

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

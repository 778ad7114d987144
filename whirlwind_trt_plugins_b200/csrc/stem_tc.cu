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
//                       of the octet's channels into a ring of 2..8 slots with
//                       TMA box copies (16-byte cp.async copies when the
//                       features do not suit TMA; zero fill outside the image);
//                       completion is counted on an mbarrier.
//   producers (8 warps) compute the octet's correlation (fused mode) on the
//                       warp-level tensor cores (mma.sync, fp32 accumulation;
//                       see corr_task_mma) or gather it from a volume tensor
//                       (volume mode) into the volume buffer in the UMMA
//                       K-major layout
//                           [group octet][d' = d+1][w' = w-w0+1][8 groups x fp16]
//   MMA (1 warp)        for each 128-voxel M-block (16 disparities x 8 columns)
//                       and K-step (two 8-group octets of one or two (kd, kw)
//                       taps) issues one tcgen05.mma with N = 3 * Cout: the three
//                       kh taps are folded into N, so one instruction adds volume
//                       row u's contribution to output rows u+1, u, u-1.  The
//                       (kd, kw) taps are start-address shifts of the same buffer.
//   epilogue (4 warps)  when output row u-1 is complete, read its accumulators
//                       out of tensor memory (releasing the slot at once: the
//                       MMA warp restarts it with accumulate = 0), add the
//                       bias, apply the activation and store fp16.
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
// MMAs accumulating into the same columns back to back cost ~150 cycles each,
// so one thread issues a row's MMAs with the M-blocks interleaved inside each
// K-step; descriptors come from kernel parameters (constant bank, uniform
// registers), never from shared memory, so the issue path does not queue
// behind the producers' loads.
//
// Synchronisation (mbarriers, every wait bounded):
//   stage_full[ns]  loader (TMA bytes or cp.async completion) -> producers
//   stage_empty[ns] producers (one arrival per warp and job) -> loader
//   vol_full[nv]    producers -> MMA        volume buffer ready
//   vol_empty[nv]   MMA (commit) -> producers   all MMAs reading it finished
// (nv = 2 or 3 volume buffers: with three, the producers run up to two rows
// ahead of the MMA warp, which hides the rows they produce while the tensor
// core's operand reads hold the shared memory.)
//   acc_full        MMA (commit) -> epilogue    row u-1 complete in every M-block
//   acc_empty       epilogue -> MMA             row u-1's slots read out (every M-block)
// A wait that expires records an error code in the device error word; the
// waiting role stops, the others run into their own bounded waits, and the
// CTA winds down and frees its tensor memory.

#include "int_div.cuh"
#include "tensor_map.cuh"
#include "umma.cuh"
#include "ww_common.cuh"

#include <algorithm>
#include <atomic>
#include <mutex>

namespace ww {


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
// Staged left columns with nt column tiles per CTA: [w0 - 8, w0 + 16) for
// one tile; for two, [w0 - 8, w0 + 32), 40 rather than the 32 needed, so the
// 80-byte rows keep the 8 channel rows of each transposing ldmatrix in
// distinct 16-byte bank groups (64-byte rows: 4-way conflicts, measured
// 3.6x the shared-memory bank conflicts).
__host__ __device__ constexpr int lstage_w(int nt) { return nt == 2 ? 40 : kLStageW; }
constexpr int kLRowBytes = kLStageW * 2;
constexpr int kMaxSteps = 32;      // K-steps per M-block (group octets <= 7)
constexpr int kMaxSlots = 8;       // staging ring depth
constexpr int kMaxVBuf = 3;        // volume row buffers
constexpr int kMaxTasks = 24;      // producer tasks per staging job (two right tiles each)
constexpr int kGroupMinMB = 4;     // M-blocks from which a row is issued and drained as two groups
constexpr bool kDualTiles = true;  // two 8-column tiles per CTA where tensor memory holds them
constexpr int kMaxFItems = 10 * 24;  // CUDA-core correlation items per job (10 columns x ceil(D/8) + 2 tiles)
// M-blocks the epilogue drains (tensor memory -> registers, slot released)
// before it stores any of them.  The MMA warp needs every M-block's slot
// back before the first K-step of the next row, so a row with more M-blocks
// than this waits for the stores of the first group: with Cout = 16 the
// packed results are small enough to drain five M-blocks (D <= 80) at once.
template <int COUTP>
constexpr int drain_blocks() { return COUTP <= 16 ? 5 : 3; }

struct StemParams {
    const __half* vol;    // volume mode: [B, G, D, H, W]
    const __half* left;   // fused mode:  [B, C, in_rows, W]
    const __half* right;
    const __half* w;      // [Cout, G, 27]
    const __half* bias;   // [Cout]
    __half* out;          // [B, Cout, D, out_rows, W]
    int* err;
    int B, C, G, H, W, D, Cout, act;   // D: disparities of this launch's band
    int d_off, D_tot;         // band start, disparities of the whole volume (output [B, Cout, D_tot, ...])
    int d_lo, d_hi;           // band-relative disparities whose volume planes are filled: [-1 or 0, D or D + 1)
    int n8;                   // right-column runs of 8 staged per job: ceil(d_hi / 8)
    int in_row0, in_rows, out_row0, out_rows;
    int Cg, KG, Dp, n_mb, nsteps, strip, n_strips, n_wtiles;
    float inv_cg;
    int vec_ok;
    int rstage_w;             // staged right columns
    int n_slots;              // staging ring depth (2..kMaxSlots)
    int n_vbuf;               // volume row buffers (2..kMaxVBuf)
    int n_tiles;              // 8-column right tiles per job: ceil(D/8) + 2
    int tpj;                  // producer tasks per job (each a range of right tiles)
    uint8_t task_jt[kMaxTasks + 1];  // task hh covers right tiles [task_jt[hh], task_jt[hh + 1])
    int raw_w_smem;           // weights staged through shared memory at set-up: 2 transposed, 1 as is, 0 not
    int use_tma;              // 1: jobs staged by TMA (else cp.async / scalar copies)
    int out_vec;              // 1: W % 8 == 0 and 16-byte aligned output (16-byte row stores)
    int n_rbox;               // right boxes of 64 columns per job
    int scale_div;            // CUDA-core correlation: 1 = sum / Cg (rounded division), 0 = sum * (1 / Cg)
    int n_grp, grp_size;      // M-block groups (1 or 2) with their own completion / release barriers
    int ntile;                // 8-column tiles per CTA (1, or 2: one M-block group per tile)
    int l_stage_w;            // staged left columns [w0 - 8, w0 + l_stage_w - 8)
    int l_row_bytes;          // 2 * l_stage_w
    uint32_t tile_vol_bytes;  // one tile's part of a volume buffer
    int n_fitems;             // CUDA-core correlation: items per job (see corr_item_fma)
    int fma_span;             // CUDA-core correlation: most jobs one producer task touches
    uint32_t tmem_cols;
    uint32_t off_b, off_vol, vol_buf_bytes, lbo_vol, off_stage, stage_slot_bytes, off_bar;
    uint32_t rbox_bytes;      // one right box: 8 Cg rows x 128 bytes
    uint32_t off_l;           // left rows within a slot
    uint32_t stage_tx;        // bytes a job's TMA copies deliver
    uint32_t off_zero;        // 128 zero bytes (rows of absent channels)
    uint32_t off_bias;        // COUTP fp32 biases (zero past Cout)
    // Per K-step descriptor templates with a zero base address: A relative to a
    // volume buffer, B relative to the B image.  Read with uniform loads.
    uint64_t tmplA[kMaxSteps];
    uint64_t tmplB[kMaxSteps];
    // Per (step, chunk): weight offset of the chunk's tap and octet within an
    // output channel's [G][27] row (-1: zero-weight partner), and the number
    // of real groups in the octet.
    int step_off[2 * kMaxSteps];
    int step_gv[2 * kMaxSteps];
    // CUDA-core correlation items of a job, ordered by (right tile, volume
    // column): bits 0..3 volume column w', 4..9 right tile jt, 15 set when
    // all 8 disparities of the item lie in [0, D).
    uint16_t fitems[kMaxFItems];
    // TMA maps of the left / right features (4-D: x = W, y = row, z = channel,
    // w = batch); boxes [24] x [8 Cg] (left) and [64] x [8 Cg] (right, swizzled).
    // Volume mode: tmap_l maps the volume (5-D, encode_volume_map), boxes
    // [24 columns] x [planes] x [8 groups].
    CUtensorMap tmap_l;
    CUtensorMap tmap_r;
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

// 8x8 transpose of 32-bit elements within each group of 8 lanes (lanes
// 8g .. 8g+7): on return, e[j] of lane 8g + i is what e[i] of lane 8g + j
// held on entry.  Three butterfly rounds of 4 shuffles.
__device__ __forceinline__ void transpose8x8(uint32_t (&e)[8], int lane)
{
#pragma unroll
    for (int s = 4; s >= 1; s >>= 1) {
        const bool upper = (lane & s) != 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (i & s) continue;
            const uint32_t send = upper ? e[i] : e[i + s];
            const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, s);
            if (upper) e[i] = recv;
            else e[i + s] = recv;
        }
    }
}

// Ties registers written by tcgen05.ld to the point after tcgen05.wait::ld:
// the empty volatile asm redefines them, so no use can be scheduled above the
// wait that precedes it.
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t (&r)[N])
{
#pragma unroll
    for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// Volume column w' held by row `row` of the correlation tiles: rows 0..7 are
// w' = 1..8 (the 16-byte aligned staged left columns 8..15, read with
// ldmatrix), row 8 is w' = 0, row 9 is w' = 9; rows 10..15 are padding.
__device__ __forceinline__ int tile_row_wp(int row)
{
    return row < 8 ? row + 1 : (row == 8 ? 0 : (row == 9 ? 9 : kWtp));
}

// (x * s, y * s) (each rounded as __fmul_rn) converted to a half2 (x in the
// low half).  Two scalar multiplies: a packed f32x2 multiply of values from
// two accumulator arrays needed register moves to pair them, which made the
// correlation's tile store ~8 % of config 4's time (measured).
__device__ __forceinline__ uint32_t scale_pair(float x, float y, float s)
{
    const __half2 h2 = __floats2half2_rn(__fmul_rn(x, s), __fmul_rn(y, s));
    return *reinterpret_cast<const uint32_t*>(&h2);
}

// Scale, round and store one 16x8 tile of correlation accumulators (8 groups
// per slot) into the volume buffer vsa ([d' = d+1][w'][8 groups] rows).
// Accumulator slot s of thread t is row m + 8 (s >> 1) (volume column
// w' = tile_row_wp(row)), column 2q + (s & 1) of right tile jt (staged right
// index 8 jt + 2q + (s & 1)), i.e. disparity d = 8 ceil(D/8) - 1 + w' - index.
//
// In slot order lanes q and q + 2 of a quarter warp write the same 16-byte
// bank group (their disparities differ by 4 planes of 160 bytes), a two-way
// conflict per store; letting the lanes with q >= 2 visit a pair's slots in
// the opposite order avoided it but cost a select per stored word, which
// measured slower (config 4 at B = 16 2053 against 1997 us).
__device__ __forceinline__ void store_corr_tile(const StemParams& p, const float (&acc)[8][4], uint32_t vsa,
                                                int jt, int lane)
{
    const int m = lane >> 2, q = lane & 3;
    const int dbase = 8 * (p.n_tiles - 2) - 1;
    const float inv_cg = p.inv_cg;
#pragma unroll
    for (int pr = 0; pr < 2; ++pr) {  // slots 2 pr, 2 pr + 1: one volume column, two right columns
        const int wp = tile_row_wp(m + 8 * pr);
        uint32_t h[2][4];
#pragma unroll
        for (int s2 = 0; s2 < 2; ++s2)
#pragma unroll
            for (int k = 0; k < 4; ++k)
                h[s2][k] = scale_pair(acc[2 * k][2 * pr + s2], acc[2 * k + 1][2 * pr + s2], inv_cg);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const int d = dbase + wp - (8 * jt + 2 * q + t);
            if (wp < kWtp && d >= p.d_lo && d < p.d_hi)
                st_shared_v4(vsa + static_cast<uint32_t>(((d + 1) * kWtp + wp) * 16), h[t][0], h[t][1], h[t][2],
                             h[t][3]);
        }
    }
}

// Staged layout of one job (slot base 1024-byte aligned; row r = e * Cg + c
// is channel c of group e of the octet):
//   right: n_rbox boxes of [8 Cg rows][64 fp16] (128-byte rows, 128-byte TMA
//          swizzle: 16-byte chunk j of row r sits at chunk j ^ (r & 7)), box k
//          holding staged right columns [64 k, 64 k + 64) = image columns
//          w0 - 8 ceil(D/8) + 64 k + ...
//   left:  at off_l, [8 Cg rows][24 fp16] (48-byte rows), image columns
//          w0 - 8 .. w0 + 15.
// Address of the 16-byte right chunk holding staged columns [8 jt, 8 jt + 8)
// of row r, given rb = slot + r * 128:
__device__ __forceinline__ uint32_t rchunk(uint32_t rb, int r, int jt, uint32_t rbox_bytes)
{
    return rb + static_cast<uint32_t>(jt >> 3) * rbox_bytes + ((static_cast<uint32_t>((jt & 7) ^ (r & 7))) << 4);
}

// Group-wise correlation of one staging job (the 8 groups of a group octet,
// one volume row) for right-column tiles [jt0, jt1), on the warp-level
// tensor cores.  Per group the band is a small GEMM
//     P[x][x'] = sum_c L[c][x] * R[c][x']          vol[d][x] = P[x][x - d] / Cg
// with M = the 10 volume columns x (w' = 0..9, padded to 16 rows), K = the
// group's channels and N = 8 staged right columns x'.  Thread t of the warp
// holds the same four (x, x') accumulator slots for every group of the
// octet, so each slot it owns becomes one 16-byte row of the volume buffer
// (8 groups of one (d, w') position) written with a single vector store.
// Products of fp16 values are exact in fp32; the tensor core adds the Cg
// products in its own order, so a volume value can differ from the CorrVolume
// kernels' sequential fp32 fma chain in the last fp32 bits (and, rarely, by
// one fp16 ulp after rounding).
// KM = 8: Cg <= 8 (m16n8k8); KM = 16: 8 < Cg <= 16 (m16n8k16).  FULL: Cg ==
// KM (no absent channels); otherwise channels >= Cg read zeros (A:
// predicated loads; B: a zeroed 128-byte row).
// tl: the CTA's column tile (its left columns start 8 tl further right, and
// its right tile jt is staged tile jt + tl).
template <int KM, bool FULL, int NT>
__device__ __forceinline__ void corr_task_mma(const StemParams& p, uint32_t slot, uint32_t zero_row,
                                              uint32_t vsa, int jt0, int jt1, int lane, int tl)
{
    constexpr int LRB = 2 * lstage_w(NT);  // staged left row bytes
    if constexpr (NT == 1) tl = 0;
    constexpr int NA = KM == 8 ? 2 : 4;  // A registers per group
    constexpr int NB = KM == 8 ? 1 : 2;  // B registers per group and tile
    constexpr int NI = KM == 8 ? 2 : 4;  // ldmatrix.x4 per tile
    const int m = lane >> 2, q = lane & 3;
    const int Cg = p.Cg;
    const uint32_t lslot = slot + p.off_l;

    // A fragments (rows = volume columns, see tile_row_wp; k = channels).
    // Rows 0..7 are the aligned staged left columns 8..15: one transposing
    // ldmatrix per 8x8 (group, channel half) matrix, absent channels reading
    // the zero row.  Rows 8 and 9 (staged columns 7 and 16) are loaded by the
    // lanes that hold them; rows 10..15 are zero.
    uint32_t a[8][NA];
    {
        const int mi = lane >> 3, rr = lane & 7;
#pragma unroll
        for (int j = 0; j < NA * 2; ++j) {  // KM 8: 2 loads of 4 groups; KM 16: 4 loads of 2 groups x 2 halves
            const int e = KM == 8 ? 4 * j + mi : 2 * j + (mi >> 1);
            const int c = KM == 8 ? rr : 8 * (mi & 1) + rr;
            const uint32_t addr = (FULL || c < Cg)
                                      ? lslot + static_cast<uint32_t>((e * Cg + c) * LRB + 16 + 16 * tl)
                                      : zero_row;
            uint32_t r4[4];
            ldmatrix_x4_trans(addr, r4);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                if (KM == 8) a[4 * j + k][0] = r4[k];
                else a[2 * j + (k >> 1)][2 * (k & 1)] = r4[k];
            }
        }
        const int col = (m == 0 ? 7 : 16) + 8 * tl;  // staged left column of row 8 + m
#pragma unroll
        for (int e = 0; e < 8; ++e) {
#pragma unroll
            for (int r = 1; r < NA; r += 2) {
                const int c0 = 2 * q + 8 * (r >> 1);
                const uint32_t la = lslot + static_cast<uint32_t>((e * Cg + c0) * LRB + 2 * col);
                const unsigned short lo = (m < 2 && (FULL || c0 < Cg)) ? ld_shared_u16(la) : 0;
                const unsigned short hi = (m < 2 && (FULL || c0 + 1 < Cg)) ? ld_shared_u16(la + LRB) : 0;
                a[e][r] = pack_b16x2(lo, hi);
            }
        }
    }

    // ldmatrix row of this lane: matrix i = lane / 8 is (group, k-half), its
    // row lane % 8 a channel.
    const int mi = lane >> 3, rr = lane & 7;
    uint32_t rb[NI];
    int rrow[NI];
#pragma unroll
    for (int k = 0; k < NI; ++k) {
        const int e = KM == 8 ? 4 * k + mi : 2 * k + (mi >> 1);
        const int c = KM == 8 ? rr : 8 * (mi & 1) + rr;
        rrow[k] = (FULL || c < Cg) ? e * Cg + c : -1;
        rb[k] = rrow[k] >= 0 ? slot + static_cast<uint32_t>(rrow[k]) * 128u : zero_row;
    }

    for (int jt = jt0; jt < jt1; ++jt) {
        __syncwarp();
        uint32_t b[8][NB];
#pragma unroll
        for (int k = 0; k < NI; ++k) {
            uint32_t r4[4];
            const uint32_t addr = (FULL || rrow[k] >= 0) ? rchunk(rb[k], rrow[k], jt + tl, p.rbox_bytes)
                                                         : rb[k] + (static_cast<uint32_t>((jt + tl) & 7) << 4);
            ldmatrix_x4_trans(addr, r4);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                if (KM == 8) b[4 * k + i][0] = r4[i];
                else b[2 * k + (i >> 1)][i & 1] = r4[i];
            }
        }
        float acc[8][4];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
#pragma unroll
            for (int s = 0; s < 4; ++s) acc[e][s] = 0.0f;
            if (KM == 8) mma_16x8x8_f16f32(acc[e], a[e][0], a[e][1], b[e][0]);
            else mma_16x8x16_f16f32(acc[e], a[e][0], a[e][1], a[e][2], a[e][3], b[e][0], b[e][NB - 1]);
        }
        store_corr_tile(p, acc, vsa, jt, lane);
    }
}

// Cg > 16: the channels run through the tensor core in chunks of 16 (the
// last one zero-padded), with the fragments of each chunk loaded per tile.
__device__ __forceinline__ void corr_task_mma_wide(const StemParams& p, uint32_t slot, uint32_t zero_row,
                                                   uint32_t vsa, int jt0, int jt1, int lane)
{
    constexpr int tl = 0;          // Cg > 16: one column tile per CTA
    constexpr int LRB = 2 * kLStageW;
    const int m = lane >> 2, q = lane & 3;
    const int mi = lane >> 3, rr = lane & 7;
    const int Cg = p.Cg;
    const uint32_t lslot = slot + p.off_l;
    for (int jt = jt0; jt < jt1; ++jt) {
        float acc[8][4];
#pragma unroll
        for (int e = 0; e < 8; ++e)
#pragma unroll
            for (int s = 0; s < 4; ++s) acc[e][s] = 0.0f;
        for (int kc = 0; kc < Cg; kc += 16) {
            __syncwarp();
            uint32_t b[8][2];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int e = 2 * k + (mi >> 1);
                const int c = kc + 8 * (mi & 1) + rr;
                const int r = e * Cg + c;
                uint32_t r4[4];
                ldmatrix_x4_trans(c < Cg ? rchunk(slot + static_cast<uint32_t>(r) * 128u, r, jt + tl, p.rbox_bytes)
                                         : zero_row + (static_cast<uint32_t>((jt + tl) & 7) << 4),
                                  r4);
#pragma unroll
                for (int i = 0; i < 4; ++i) b[2 * k + (i >> 1)][i & 1] = r4[i];
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                uint32_t a[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    // row m (r even) or 8 + m (r odd) of the tile: see tile_row_wp
                    const int c0 = kc + 2 * q + 8 * (r >> 1);
                    const bool top = (r & 1) == 0;
                    const int col = (top ? m + 8 : (m == 0 ? 7 : 16)) + 8 * tl;
                    const bool row_ok = top || m < 2;
                    const uint32_t la = lslot + static_cast<uint32_t>((e * Cg + c0) * LRB + 2 * col);
                    const unsigned short lo = (row_ok && c0 < Cg) ? ld_shared_u16(la) : 0;
                    const unsigned short hi = (row_ok && c0 + 1 < Cg) ? ld_shared_u16(la + LRB) : 0;
                    a[r] = pack_b16x2(lo, hi);
                }
                mma_16x8x16_f16f32(acc[e], a[0], a[1], a[2], a[3], b[e][0], b[e][1]);
            }
        }
        store_corr_tile(p, acc, vsa, jt, lane);
    }
}

// One volume row's MMAs: K-step 0 restarts output row u+1 in its slot sn of
// every M-block (accumulate = 0 for that slot, the other two accumulate),
// K-steps 1..S-1 add into all three slots, the NMB M-blocks interleaved inside
// each step.  NMB is a compile-time constant: a runtime M-block loop around
// each MMA cut the issue rate by about 40 % (measured).
template <int COUTP, int NMB>
__device__ __forceinline__ void issue_row(const StemParams& p, uint32_t tmem_base, uint64_t a0, uint64_t b0,
                                          int sn)
{
    constexpr int N = 3 * COUTP;
    constexpr uint32_t idesc = idesc_f16_f32(128, N);
    constexpr uint32_t idesc1 = idesc_f16_f32(128, COUTP);      // one slot
    constexpr uint32_t idesc2 = idesc_f16_f32(128, 2 * COUTP);  // two adjacent slots
    constexpr uint64_t mb_step = (16 * kWtp * 16) >> 4;         // one M-block along D
    constexpr uint64_t blk = (COUTP * 16) >> 4;                 // one slot of B rows
    {
        const uint64_t a = p.tmplA[0] + a0, bd = p.tmplB[0] + b0;
#pragma unroll
        for (int m = 0; m < NMB; ++m) {
            const uint32_t d = tmem_base + m * N;
            const uint64_t am = a + m * mb_step;
            mma_f16_ss(d + sn * COUTP, am, bd + sn * blk, idesc1, 0);
            if (sn == 0) mma_f16_ss(d + COUTP, am, bd + blk, idesc2, 1);
            else if (sn == 2) mma_f16_ss(d, am, bd, idesc2, 1);
            else {
                mma_f16_ss(d, am, bd, idesc1, 1);
                mma_f16_ss(d + 2 * COUTP, am, bd + 2 * blk, idesc1, 1);
            }
        }
    }
    for (int st = 1; st < p.nsteps; ++st) {
        const uint64_t a = p.tmplA[st] + a0, bd = p.tmplB[st] + b0;
#pragma unroll
        for (int m = 0; m < NMB; ++m) mma_f16_ss(tmem_base + m * N, a + m * mb_step, bd, idesc, 1);
    }
}

template <int COUTP>
__device__ __forceinline__ void issue_row_n(const StemParams& p, uint32_t tmem_base, uint64_t a0, uint64_t b0,
                                            int sn, int nmb)
{
    // M-block counts the tensor memory holds: NMB * 3 * COUTP <= 512.
    switch (nmb) {
#define WW_ISSUE_CASE(NMB) \
    case NMB:              \
        if constexpr (NMB * 3 * COUTP <= 512) issue_row<COUTP, NMB>(p, tmem_base, a0, b0, sn); \
        break;
        WW_ISSUE_CASE(1) WW_ISSUE_CASE(2) WW_ISSUE_CASE(3) WW_ISSUE_CASE(4) WW_ISSUE_CASE(5)
        WW_ISSUE_CASE(6) WW_ISSUE_CASE(7) WW_ISSUE_CASE(8) WW_ISSUE_CASE(9) WW_ISSUE_CASE(10)
#undef WW_ISSUE_CASE
        default: break;
    }
}

// Group-wise correlation of one item of a staging job on the CUDA cores:
// item (volume column w', right tile jt, group half q) is, for the groups
// e = 4q .. 4q+3 of the octet, the 8 disparities d = 8 ceil(D/8) - 1 + w' - x'
// of the staged right columns x' = 8 jt .. 8 jt + 7:
//     vol[e][d][w'] = round_fp16(scale(sum_c L[e Cg + c][w'] * R[e Cg + c][x']))
// summed as one fp32 fma chain in channel order, c = 0 .. Cg-1, from +0 (the
// fp16 products are exact in fp32) and scaled as ww_corr_volume scales the
// same call (scale_div: / Cg, else * (1 / Cg)): the same value, bit for bit,
// as ww_corr_volume's.  Per (channel, group) a lane reads one
// 16-byte chunk of right columns and one left value and does 8 fmas into
// acc[group][x' - 8 jt]; the 4 groups of a disparity are then one 8-byte
// half of a 16-byte volume row.  The lanes of a quarter warp take
// consecutive columns w' of one tile, so their right reads are one
// broadcast and their volume rows (11 rows apart between neighbouring w' at
// equal x') fall in distinct bank groups.  CG > 0: Cg known at compile time.
template <int CG>
__device__ __forceinline__ void corr_item_fma(const StemParams& p, const uint8_t* stage, uint8_t* vol, int item,
                                              int q)
{
    const int ent = p.fitems[item];
    const int wp = ent & 15, jt = (ent >> 4) & 63;
    const bool full = (ent & 0x8000) != 0;
    const int Cg = CG > 0 ? CG : p.Cg;
    // Right chunk of staged columns [8 jt, 8 jt + 8) in row r: box jt / 8,
    // 16-byte chunk (jt % 8) ^ (r % 8) of the row (128-byte TMA swizzle).
    const uint8_t* rbox = stage + (jt >> 3) * p.rbox_bytes + 4 * q * Cg * 128;
    const uint32_t jsw = static_cast<uint32_t>(jt & 7);
    constexpr int LRB = 2 * kLStageW;  // the CUDA-core engine runs one column tile per CTA
    const uint8_t* lcol = stage + p.off_l + 2 * (wp + 7) + 4 * q * Cg * LRB;  // staged column w' + 7
    const int rq = 4 * q * Cg;  // first row of the half
    float acc[4][8];
#pragma unroll
    for (int e = 0; e < 4; ++e)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[e][j] = 0.0f;
#pragma unroll(CG > 0 ? CG : 1)
    for (int c = 0; c < Cg; ++c) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int rl = e * Cg + c;  // row within the half
            const uint32_t sw = ((jsw ^ static_cast<uint32_t>((rq + rl) & 7)) << 4);
            const uint4 rv = *reinterpret_cast<const uint4*>(rbox + rl * 128 + sw);
            const unsigned short lv = *reinterpret_cast<const unsigned short*>(lcol + rl * LRB);
            unsigned short h[8];
            unpack_b16x2(rv.x, h[0], h[1]);
            unpack_b16x2(rv.y, h[2], h[3]);
            unpack_b16x2(rv.z, h[4], h[5]);
            unpack_b16x2(rv.w, h[6], h[7]);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[e][j] = fma_f16f16f32(lv, h[j], acc[e][j]);
        }
    }
    const int d0 = 8 * (p.n_tiles - 2) - 1 + wp - 8 * jt;  // disparity of x' = 8 jt
    uint8_t* row0 = vol + ((d0 + 1) * kWtp + wp) * 16 + 8 * q;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int d = d0 - j;
        if (full || (d >= p.d_lo && d < p.d_hi)) {
            uint2 v;
            if (p.scale_div) {
                const __half2 h01 = __floats2half2_rn(div_int(acc[0][j], Cg, p.inv_cg), div_int(acc[1][j], Cg, p.inv_cg));
                const __half2 h23 = __floats2half2_rn(div_int(acc[2][j], Cg, p.inv_cg), div_int(acc[3][j], Cg, p.inv_cg));
                v.x = *reinterpret_cast<const uint32_t*>(&h01);
                v.y = *reinterpret_cast<const uint32_t*>(&h23);
            } else {
                v.x = scale_pair(acc[0][j], acc[1][j], p.inv_cg);
                v.y = scale_pair(acc[2][j], acc[3][j], p.inv_cg);
            }
            *reinterpret_cast<uint2*>(row0 - j * kWtp * 16) = v;
        }
    }
}

// Correlation variants (a kernel template parameter, so each instantiation
// carries only its own producer path).  Warp-level tensor cores: 1: Cg == 8,
// 2: Cg < 8, 3: Cg == 16, 4: 8 < Cg < 16, 5: Cg > 16.  CUDA cores
// (corr_item_fma): 6: Cg == 8, 7: Cg == 4, 8: Cg == 12, 9: Cg == 16, 10: any.
template <int CORR, int NT>
__device__ __forceinline__ void corr_task(const StemParams& p, uint32_t slot, uint32_t zero_row, uint32_t vsa,
                                          int jt0, int jt1, int lane, int tl)
{
    if constexpr (CORR == 1) corr_task_mma<8, true, NT>(p, slot, zero_row, vsa, jt0, jt1, lane, tl);
    else if constexpr (CORR == 2) corr_task_mma<8, false, NT>(p, slot, zero_row, vsa, jt0, jt1, lane, tl);
    else if constexpr (CORR == 3) corr_task_mma<16, true, NT>(p, slot, zero_row, vsa, jt0, jt1, lane, tl);
    else if constexpr (CORR == 4) corr_task_mma<16, false, NT>(p, slot, zero_row, vsa, jt0, jt1, lane, tl);
    else corr_task_mma_wide(p, slot, zero_row, vsa, jt0, jt1, lane);
}

template <int CORR>
__device__ __forceinline__ void corr_item(const StemParams& p, const uint8_t* stage, uint8_t* vol, int item, int q)
{
    if constexpr (CORR == 6) corr_item_fma<8>(p, stage, vol, item, q);
    else if constexpr (CORR == 7) corr_item_fma<4>(p, stage, vol, item, q);
    else if constexpr (CORR == 8) corr_item_fma<12>(p, stage, vol, item, q);
    else if constexpr (CORR == 9) corr_item_fma<16>(p, stage, vol, item, q);
    else corr_item_fma<0>(p, stage, vol, item, q);
}

// Correlation engine of the fused kernel (WW_CORR_ENGINE_*), process-wide.
std::atomic<int> g_corr_engine{WW_CORR_ENGINE_TENSOR};

inline int corr_variant(int Cg, bool cuda_cores)
{
    if (cuda_cores) return Cg == 8 ? 6 : Cg == 4 ? 7 : Cg == 12 ? 8 : Cg == 16 ? 9 : 10;
    return Cg == 8 ? 1 : Cg < 8 ? 2 : Cg == 16 ? 3 : Cg < 16 ? 4 : 5;
}

// CORR: correlation variant (fused mode; 0 in volume mode).
// NT: 8-column tiles per CTA (2 only for Cout <= 16 with the tensor-core
// correlation variants 1-4).
template <int COUTP, bool FUSED, int CORR, int NT>
__global__ void __launch_bounds__(kThreads, 1) stem_tc_kernel(const __grid_constant__ StemParams p)
{
    extern __shared__ __align__(1024) uint8_t smem[];
    constexpr int NR = 5 * COUTP;      // rows of the rotated B image
    constexpr int N = 3 * COUTP;       // MMA N
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // ---- tile coordinates ----
    // Adjacent column tiles of one strip are consecutive CTAs, so they run
    // at the same time: the halves of each 32-byte output sector that two
    // neighbouring tiles write meet in L2, and so do their overlapping
    // right-feature windows.
    int t = blockIdx.x;
    const int wt = t % p.n_wtiles;
    t /= p.n_wtiles;
    const int strip = t % p.n_strips;
    const int b = t / p.n_strips;
    const int w0 = wt * kWt * NT;
    const int r0 = p.out_row0 + strip * p.strip;                    // first output row
    const int r1 = min(r0 + p.strip, p.out_row0 + p.out_rows);     // one past last
    const int u_first = r0 - 1;
    const int n_iter = (r1 - r0) + 2;                              // volume rows u_first .. r1
    // volume rows inside the image (a contiguous range) and the staging jobs over them
    const int uv0 = max(u_first, 0);
    const int uv1 = min(u_first + n_iter, p.H);
    const int total_jobs = (FUSED || p.use_tma) ? max(0, uv1 - uv0) * p.KG : 0;

    uint8_t* sB = smem + p.off_b;
    uint8_t* sVol = smem + p.off_vol;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_bar);
    const int NV = p.n_vbuf;
    uint64_t* vol_full = bars;                        // [NV]
    uint64_t* vol_empty = bars + kMaxVBuf;            // [NV]
    uint64_t* final_bar = bars + 2 * kMaxVBuf;
    uint64_t* stage_full = final_bar + 1;             // [n_slots]
    uint64_t* stage_empty = stage_full + p.n_slots;   // [n_slots]
    uint64_t* acc_full = stage_empty + p.n_slots;     // [2]: one per M-block group
    uint64_t* acc_empty = acc_full + 2;               // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

    // ---- set-up: barriers, TMEM, B image, zeroed volume buffers ----
    if (threadIdx.x == 0) {
        for (int i = 0; i < NV; ++i) {
            mbar_init(smem_addr(&vol_full[i]), kProdWarps);
            mbar_init(smem_addr(&vol_empty[i]), 1);
        }
        for (int i = 0; i < p.n_slots; ++i) {
            mbar_init(smem_addr(&stage_full[i]), p.use_tma ? 1 : 32);
            mbar_init(smem_addr(&stage_empty[i]), kProdWarps);
        }
        mbar_init(smem_addr(final_bar), 1);
        for (int g = 0; g < 2; ++g) {
            mbar_init(smem_addr(&acc_full[g]), 1);
            mbar_init(smem_addr(&acc_empty[g]), kEpiWarps);
        }
        mbar_fence_init();
    }
    if (warp == kMmaWarp) tmem_alloc(smem_addr(tmem_slot), p.tmem_cols);

    // Weights [Cout][G][27] fp16 are first staged into shared memory (the
    // volume region, unused until set-up ends) and the B image is gathered
    // from there.  raw_w_smem == 2 (G a multiple of 8): staged transposed to
    // [Cout][27][G], so the 8 groups of an entry are one aligned 16-byte
    // load; the lanes of a warp take consecutive (o, g) rows, so their 2-byte
    // global loads cover one contiguous block and their shared stores are
    // consecutive halves (no bank conflicts).  raw_w_smem == 1: copied as is
    // with 16-byte cp.async, gathered with 2-byte loads.  0: gathered from
    // global memory.
    const int wmode = p.raw_w_smem;
    const uint32_t raw = smem_addr(sVol);
    if (wmode == 2) {
        const unsigned short* wg = reinterpret_cast<const unsigned short*>(p.w);
        const int G = p.G;
        for (int r = threadIdx.x; r < p.Cout * G; r += kThreads) {
            const int o = r / G, g = r - o * G;
            const unsigned short* src = wg + static_cast<size_t>(r) * 27;
            const uint32_t dst = raw + 2u * static_cast<uint32_t>(o * 27 * G + g);
#pragma unroll
            for (int t = 0; t < 27; ++t) st_shared_u16(dst + 2u * static_cast<uint32_t>(t * G), __ldg(src + t));
        }
        __syncthreads();
    } else if (wmode == 1) {
        const uint32_t wbytes = static_cast<uint32_t>(p.Cout * p.G * 54);
        for (uint32_t i = threadIdx.x * 16; i < wbytes; i += kThreads * 16)
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n"
                         :
                         : "r"(raw + i), "l"(reinterpret_cast<const uint8_t*>(p.w) + i)
                         : "memory");
        asm volatile("cp.async.wait_all;\n" ::: "memory");
        __syncthreads();
    }
    // TMA staging of job j (volume row uv0 + j / KG, group octet j % KG) into
    // slot j % n_slots: one elected lane arms stage_full with the byte count
    // and issues n_rbox right boxes and one left box (zero fill outside the
    // image and past the last channel).  Volume mode: one box of the volume,
    // [8 groups][planes d_lo .. d_hi - 1][columns w0 - 8 .. w0 + 15] (zero
    // fill outside the image and past the last group).
    // The ring position (slot, row offset jr = j / KG, octet kg = j % KG) is
    // passed in: the loops keep it as running counters, without a division
    // per job.
    const int n_runs = p.n8;
    auto tma_job = [&](int slot, int jr, int kg) {
        const uint32_t sbase = smem_addr(smem + p.off_stage + slot * p.stage_slot_bytes);
        const uint32_t full = smem_addr(&stage_full[slot]);
        mbar_arrive_expect_tx(full, p.stage_tx);
        if constexpr (FUSED) {
            const int urow = uv0 + jr - p.in_row0;
            const int c0 = kg * 8 * p.Cg;
            for (int k = 0; k < p.n_rbox; ++k)
                tma_load_4d(sbase + k * p.rbox_bytes, &p.tmap_r, w0 - 8 * n_runs - p.d_off + 64 * k, urow, c0, b,
                            full);
            tma_load_4d(sbase + p.off_l, &p.tmap_l, w0 - 8, urow, c0, b, full);
        } else {
            tma_load_5d(sbase, &p.tmap_l, w0 - 8, uv0 + jr, p.d_off + p.d_lo, 8 * kg, b, full);
        }
    };
    // The first n_slots jobs need no free slot: issue them now, so their
    // loads overlap the B image build (the staging ring is not touched by
    // set-up; the barriers are initialised and visible after the sync above).
    const int n_pre = (p.use_tma && wmode != 0) ? min(p.n_slots, total_jobs) : 0;
    if (n_pre > 0 && warp == kLoadWarp) {
        if (elect_one())
            for (int j = 0; j < n_pre; ++j) tma_job(j, j / p.KG, j % p.KG);
        __syncwarp();
    }
    // B image: entry (step s, chunk c, row n = blk * COUTP + o) holds the 8
    // fp16 weights of the chunk's group octet for output channel o and tap
    // (kd, kh, kw); blocks blk = 0..4 are [kh2, kh1, kh0, kh2, kh1].  The
    // host precomputes each chunk's tap offset (step_off = 216 kg + 9 kd + kw;
    // -1 for a zero-weight partner) and valid group count (step_gv).
    if (wmode == 2) {
        // One item per (chunk, kh, o): one 16-byte load, stored to the one or
        // two blocks of that kh.
        const int G = p.G;
        for (int i = threadIdx.x; i < p.nsteps * 2 * 3 * COUTP; i += kThreads) {
            const int o = i % COUTP, r2 = i / COUTP;
            const int kh = r2 % 3, sc = r2 / 3;
            const int toff = p.step_off[sc], gv = p.step_gv[sc];
            uint32_t v[4] = {0u, 0u, 0u, 0u};
            if (toff >= 0 && o < p.Cout) {
                const int kg = toff / 216, tap = toff - kg * 216 + kh * 3;
                ld_shared_v4(raw + 2u * static_cast<uint32_t>((o * 27 + tap) * G + 8 * kg), v);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    if (2 * q >= gv) v[q] &= 0xFFFF0000u;
                    if (2 * q + 1 >= gv) v[q] &= 0x0000FFFFu;
                }
            }
            const int blk0 = 2 - kh;  // kh2 -> 0 (and 3), kh1 -> 1 (and 4), kh0 -> 2
            st_shared_v4(smem_addr(sB) + 16u * static_cast<uint32_t>((sc * 5 + blk0) * COUTP + o), v[0], v[1],
                         v[2], v[3]);
            if (kh > 0)
                st_shared_v4(smem_addr(sB) + 16u * static_cast<uint32_t>((sc * 5 + blk0 + 3) * COUTP + o), v[0],
                             v[1], v[2], v[3]);
        }
    } else {
        const unsigned short* wg = reinterpret_cast<const unsigned short*>(p.w);
        const int g27 = p.G * 27;
        for (int i = threadIdx.x; i < p.nsteps * 2 * NR; i += kThreads) {
            const int n = i % NR, sc = i / NR;
            const int blk = n / COUTP, o = n - blk * COUTP;
            const int kh = (blk == 2) ? 0 : ((blk == 1 || blk == 4) ? 1 : 2);
            const int toff = p.step_off[sc], gv = p.step_gv[sc];
            uint32_t v[4] = {0u, 0u, 0u, 0u};
            if (toff >= 0 && o < p.Cout) {
                const int base = o * g27 + kh * 3 + toff;
                unsigned short h[8];
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    h[e] = e < gv ? (wmode == 1 ? ld_shared_u16(raw + 2u * static_cast<uint32_t>(base + e * 27))
                                                : wg[base + e * 27])
                                  : static_cast<unsigned short>(0);
#pragma unroll
                for (int q = 0; q < 4; ++q) v[q] = pack_b16x2(h[2 * q], h[2 * q + 1]);
            }
            st_shared_v4(smem_addr(sB) + 16u * static_cast<uint32_t>(i), v[0], v[1], v[2], v[3]);
        }
    }
    __syncthreads();  // the staged weights are consumed before the region is zeroed
    // Both volume buffers start as zeros: halo planes and padding stay zero;
    // so do the zero rows that stand in for absent channels.
    for (uint32_t i = threadIdx.x * 16; i < NV * p.vol_buf_bytes; i += kThreads * 16)
        *reinterpret_cast<uint4*>(sVol + i) = make_uint4(0, 0, 0, 0);
    for (uint32_t i = threadIdx.x * 16; i < 128u; i += kThreads * 16)
        *reinterpret_cast<uint4*>(smem + p.off_zero + i) = make_uint4(0, 0, 0, 0);
    if (threadIdx.x < COUTP)
        reinterpret_cast<float*>(smem + p.off_bias)[threadIdx.x] =
            threadIdx.x < p.Cout ? __half2float(p.bias[threadIdx.x]) : 0.0f;

    fence_proxy_async_smem();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem_base = *tmem_slot;

    if (warp < kEpiWarps) {
        // Zero this quadrant's lanes of every accumulator column.
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(warp * 32) << 16);
        const uint32_t zeros[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int c = 0; c < NT * p.n_mb * N; c += 8) tmem_st8(lane_base + c, zeros);
        tmem_wait_st();
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();

    if (warp < kEpiWarps) {
        // ======================= epilogue =======================
        // Per volume row: first drain the completed output row of up to
        // kDrain M-blocks (tensor-memory load, bias + activation, fp16 pack,
        // zero the slot, release it with acc_empty), so the MMA warp can
        // start the next row at once; then store them.
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(warp * 32) << 16);
        constexpr int kDrain = drain_blocks<COUTP>();
        const int rr = warp * 32 + lane;  // M row
        const int dsub = rr >> 3;         // 0..15
        const float* sbias = reinterpret_cast<const float*>(smem + p.off_bias);
        const int64_t plane_out = i64(p.out_rows) * p.W;
        const int64_t ostride = i64(p.D_tot) * plane_out;
        bool ok = true;
        for (int it = 0; it < n_iter && ok; ++it) {
            const int r = u_first + it - 1;  // output row completed by this volume row
            const int slot = ((r % 3) + 3) % 3;
            // One commit per row and M-block group covers the group's
            // M-blocks: they complete together (their last K-step is issued
            // back to back), and a commit per M-block made the epilogue see
            // them ~0.3-0.5 us apart (measured).
            for (int grp = 0; grp < p.n_grp && ok; ++grp) {
            // Two tiles: group = tile, every M-block; one tile: M-block ranges.
            const int tile = NT == 2 ? grp : 0;
            const int m_beg = NT == 2 ? 0 : grp * p.grp_size;
            const int m_end = NT == 2 ? p.n_mb : min(p.n_mb, m_beg + p.grp_size);
            const int w0t = w0 + kWt * tile;  // the tile's first column
            const int w = w0t + (rr & 7);
            const uint32_t tile_cols = static_cast<uint32_t>(tile * p.n_mb * N);
            if (!warp_wait(smem_addr(&acc_full[grp]), it & 1, p.err, 1)) {
                ok = false;
                break;
            }
            fence_after_sync();
            for (int m0 = m_beg; m0 < m_end && ok; m0 += kDrain) {
                const int mcnt = min(kDrain, m_end - m0);
                uint32_t ph[kDrain][COUTP / 2];  // fp16 results, packed as (o, o + 1) pairs
                // With Cout = 16, M-blocks in pairs: both tensor-memory loads
                // in flight behind one wait (each wait costs a load latency);
                // with Cout = 32 a pair's registers would spill.
                constexpr int kPair = COUTP <= 16 ? 2 : 1;
#pragma unroll
                for (int j = 0; j < kDrain; j += kPair) {
                    if (j >= mcnt) break;
                    const bool two = kPair == 2 && j + 1 < mcnt;
                    uint32_t acc[kPair][COUTP];
#pragma unroll
                    for (int h = 0; h < kPair; ++h) {
                        if (h == 1 && !two) break;
                        const uint32_t col = lane_base + tile_cols + (m0 + j + h) * N + slot * COUTP;
#pragma unroll
                        for (int c = 0; c < COUTP; c += 16) {
                            uint32_t v16[16];
                            tmem_ld16(col + c, v16);
#pragma unroll
                            for (int q = 0; q < 16; ++q) acc[h][c + q] = v16[q];
                        }
                    }
                    tmem_wait_ld();
#pragma unroll
                    for (int h = 0; h < kPair; ++h) reg_fence(acc[h]);  // no use of acc above the wait
                    // The row's slots are free once read: the MMA warp restarts
                    // them with accumulate = 0 (no zeroing here).
                    if (m0 + j + (two ? 1 : 0) == m_end - 1) {
                        fence_before_sync();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(smem_addr(&acc_empty[grp]));
                    }
#pragma unroll
                    for (int h = 0; h < kPair; ++h) {
                        if (h == 1 && !two) break;
#pragma unroll
                        for (int k = 0; k < COUTP / 2; ++k) {
                            const float2 bb = *reinterpret_cast<const float2*>(sbias + 2 * k);
                            const __half2 h2 =
                                __floats2half2_rn(act_apply(__uint_as_float(acc[h][2 * k]) + bb.x, p.act),
                                                  act_apply(__uint_as_float(acc[h][2 * k + 1]) + bb.y, p.act));
                            ph[j + h][k] = *reinterpret_cast<const uint32_t*>(&h2);
                        }
                    }
                }
                if (!ok || r < r0 || r >= r1) continue;  // warp-uniform
                __half* orow0 = p.out + (i64(b) * p.Cout * p.D_tot + p.d_off) * plane_out + i64(r - p.out_row0) * p.W;
#pragma unroll
                for (int j = 0; j < kDrain; ++j) {
                    if (j >= mcnt) break;
                    const int d = (m0 + j) * 16 + dsub;
                    __half* orow = orow0 + i64(d) * plane_out;
                    if (p.out_vec) {
                        // The 8 lanes of a lane group hold the 8 columns of one
                        // disparity: transpose blocks of 8 o-pairs among them so
                        // each lane ends with 8 columns of two channels, written
                        // as two 16-byte rows.
#pragma unroll
                        for (int blk = 0; blk < COUTP / 16; ++blk) {
                            uint32_t e[8];
#pragma unroll
                            for (int i = 0; i < 8; ++i) e[i] = ph[j][8 * blk + i];
                            transpose8x8(e, lane);
                            const int o0 = 16 * blk + 2 * (lane & 7);
                            const uint4 lo =
                                make_uint4(__byte_perm(e[0], e[1], 0x5410), __byte_perm(e[2], e[3], 0x5410),
                                           __byte_perm(e[4], e[5], 0x5410), __byte_perm(e[6], e[7], 0x5410));
                            const uint4 hi =
                                make_uint4(__byte_perm(e[0], e[1], 0x7632), __byte_perm(e[2], e[3], 0x7632),
                                           __byte_perm(e[4], e[5], 0x7632), __byte_perm(e[6], e[7], 0x7632));
                            if (d < p.D && o0 < p.Cout && w0t < p.W) *reinterpret_cast<uint4*>(orow + o0 * ostride + w0t) = lo;
                            if (d < p.D && o0 + 1 < p.Cout && w0t < p.W)
                                *reinterpret_cast<uint4*>(orow + (o0 + 1) * ostride + w0t) = hi;
                        }
                    } else if (d < p.D && w < p.W) {
#pragma unroll
                        for (int k = 0; k < COUTP / 2; ++k) {
                            const __half2 h2 = *reinterpret_cast<const __half2*>(&ph[j][k]);
                            if (2 * k < p.Cout) orow[(2 * k) * ostride + w] = __low2half(h2);
                            if (2 * k + 1 < p.Cout) orow[(2 * k + 1) * ostride + w] = __high2half(h2);
                        }
                    }
                }
            }
            }  // M-block groups
        }
    } else if (warp == kMmaWarp) {
        // ======================= MMA issue =======================
        // Row by row: once volume row it is produced (vol_full), per M-block
        // group: once the epilogue has drained the group's slots of row it-1
        // (acc_empty[g]), issue the group's nsteps K-steps with its M-blocks
        // interleaved inside each step and commit the group (acc_full[g]).
        // With two groups the epilogue drains group 0 of a row while group
        // 1's MMAs run, and group 0 of the next row starts without waiting
        // for group 1's drain.  MMAs into the same accumulator back to back are
        // latency-bound (~150 cycles each); independent ones run at the
        // shared-memory bound (~56 cycles for M=128, N=96), which this order
        // reaches from n_mb = 3 on.  Lane 0 alone runs the loop: a warp-wide
        // elect + __syncwarp around every MMA, or a scheduler loop with
        // per-MMA bookkeeping, halve to quarter the issue rate (measured).
        if (lane == 0) {
            const uint64_t vol_base = smem_addr(sVol) >> 4;
            const uint64_t b_base = smem_addr(sB) >> 4;
            int vb = 0, vph = 0;  // buffer it % NV and its phase (it / NV) & 1, kept running
            for (int it = 0; it < n_iter; ++it, (++vb == NV ? (vb = 0, vph ^= 1) : 0)) {
                if (!wait_or_fail(smem_addr(&vol_full[vb]), vph, p.err, 2)) break;
                const int u = u_first + it;
                bool row_ok = true;
                for (int grp = 0; grp < p.n_grp; ++grp) {
                    if (it > 0 && !wait_or_fail(smem_addr(&acc_empty[grp]), (it - 1) & 1, p.err, 3)) {
                        row_ok = false;
                        break;
                    }
                    fence_after_sync();
                    if (u >= 0 && u < p.H) {  // rows outside the image issue nothing
                        const int tile = NT == 2 ? grp : 0;
                        const int m0 = NT == 2 ? 0 : grp * p.grp_size;
                        const int cnt = NT == 2 ? p.n_mb : min(p.grp_size, p.n_mb - m0);
                        const int rot = (((1 - u) % 3) + 3) % 3;
                        const uint64_t a0 = vol_base + static_cast<uint64_t>((vb * p.vol_buf_bytes) >> 4) +
                                            static_cast<uint64_t>((tile * p.tile_vol_bytes) >> 4) +
                                            static_cast<uint64_t>(m0) * ((16 * kWtp * 16) >> 4);
                        const uint64_t b0 = b_base + static_cast<uint64_t>((rot * COUTP * 16) >> 4);
                        // K-step 0 starts output row u+1 in its slot (u+1) mod 3 (it
                        // still holds the row the epilogue drained).
                        issue_row_n<COUTP>(p, tmem_base + static_cast<uint32_t>((tile * p.n_mb + m0) * 3 * COUTP), a0, b0,
                                           (u + 1) % 3, cnt);
                    }
                    mma_commit(smem_addr(&acc_full[grp]));
                }
                if (!row_ok) break;
                mma_commit(smem_addr(&vol_empty[vb]));
            }
        }
        __syncwarp();
    } else if (warp == kLoadWarp) {
        // ======================= loader =======================
        // Job j = (volume row uv0 + j / KG, group octet j % KG) -> slot j % NS,
        // in the layout described at rchunk().  With TMA: one elected lane
        // arms stage_full with the job's byte count and issues n_rbox + 1 box
        // copies (zero fill outside the image and past the last channel).
        // Otherwise (W % 8 != 0 or unaligned features) lanes copy 16-byte
        // vectors of whole channel rows with cp.async (or element by element).
        if (FUSED || p.use_tma) {
            const int Cg = p.Cg;
            const int NS = p.n_slots;
            const int rbase = w0 - 8 * n_runs - p.d_off;
            const int nvr = p.rstage_w / 8;
            int issued = n_pre;  // jobs [0, n_pre) were issued during set-up
            // Running ring position of job j: slot j % NS, round j / NS, row
            // offset j / KG, octet j % KG (no division per job).
            int slot = n_pre == NS ? 0 : n_pre, rnd = n_pre == NS ? 1 : 0;
            int jr = n_pre / p.KG, kg = n_pre - jr * p.KG;
            auto advance = [&] {
                if (++slot == NS) { slot = 0; ++rnd; }
                if (++kg == p.KG) { kg = 0; ++jr; }
            };
            for (int j = n_pre; j < total_jobs; ++j, advance()) {
                if (rnd > 0 && !warp_wait(smem_addr(&stage_empty[slot]), (rnd - 1) & 1, p.err, 6)) break;
                issued = j + 1;
                if (p.use_tma) {
                    if (elect_one()) tma_job(slot, jr, kg);
                    __syncwarp();
                    continue;
                }
                if constexpr (!FUSED) continue;  // (volume mode stages only by TMA)
                const uint32_t sbase = smem_addr(smem + p.off_stage + slot * p.stage_slot_bytes);
                const int urow = uv0 + jr - p.in_row0;
                const uint32_t full = smem_addr(&stage_full[slot]);
                for (int lc = lane; lc < 8 * Cg; lc += 32) {  // lc = row of the job (e * Cg + c)
                    const int ge = lc / Cg, cc = lc - ge * Cg;
                    const int g = kg * 8 + ge;
                    const bool gv = g < p.G;
                    const int64_t roff = ((i64(b) * p.C + (gv ? g * Cg + cc : 0)) * p.in_rows + urow) * p.W;
                    constexpr int nlv = lstage_w(NT) / 8;
                    for (int v = 0; v < nlv + nvr; ++v) {
                        const bool isL = v < nlv;
                        const int x = isL ? (w0 - 8 + 8 * v) : (rbase + 8 * (v - nlv));
                        const uint32_t dst = isL ? sbase + p.off_l + lc * (2 * lstage_w(NT)) + 16 * v
                                                 : rchunk(sbase + lc * 128u, lc, v - nlv, p.rbox_bytes);
                        const __half* srow = (isL ? p.left : p.right) + roff;
                        if (p.vec_ok) {
                            const bool in = gv && x >= 0 && x < p.W;  // whole vector (W % 8 == 0)
                            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n"
                                         :
                                         : "r"(dst), "l"(in ? srow + x : srow), "r"(in ? 16 : 0)
                                         : "memory");
                        } else {
                            __align__(16) __half h[8];
#pragma unroll
                            for (int q = 0; q < 8; ++q) {
                                const int xx = x + q;
                                h[q] = (gv && xx >= 0 && xx < p.W) ? srow[xx] : __float2half_rn(0.0f);
                            }
                            const uint4 v4 = *reinterpret_cast<const uint4*>(h);
                            st_shared_v4(dst, v4.x, v4.y, v4.z, v4.w);
                        }
                    }
                }
                if (p.vec_ok) {
                    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" : : "r"(full) : "memory");
                } else {
                    __threadfence_block();
                    mbar_arrive(full);
                }
            }
            // Nothing may still be landing in shared memory when the CTA exits:
            // wait (bounded) for the last fill of each slot, then for any
            // cp.async of this thread.
            for (int j = std::max(0, issued - NS); j < issued; ++j)
                wait_or_fail(smem_addr(&stage_full[j % NS]), (j / NS) & 1, p.err, 8);
            asm volatile("cp.async.wait_all;\n" ::: "memory");
        }
    } else {
        // ======================= producers =======================
        // Fused mode: the job of each (volume row, group octet) is split into
        // tpj tasks (ranges of right-column tiles); task tau = job * tpj + h
        // goes to producer warp tau mod kProdWarps, which runs the
        // tensor-core correlation of corr_task_mma on it.  Every warp waits on
        // and releases every job (and every volume row) in order, with or
        // without tasks in it, so no warp's parity wait can fall two phases
        // behind a barrier.  Volume mode: the warps gather the row's slice of
        // the volume tensor.
        const int pw = warp - kProdWarp0;
        const uint32_t zero_row = smem_addr(smem + p.off_zero);
        bool ok = true;
        int vb = 0, vrnd = 0;  // buffer it % NV and round it / NV, kept running
        int js = 0, jph = 0;   // slot and phase of the next staging job (jobs in order)
        auto next_job = [&] {
            if (++js == p.n_slots) { js = 0; jph ^= 1; }
        };
        for (int it = 0; it < n_iter && ok; ++it, (++vb == NV ? (vb = 0, ++vrnd) : 0)) {
            const int u = u_first + it;
            if (vrnd > 0 && !warp_wait(smem_addr(&vol_empty[vb]), (vrnd - 1) & 1, p.err, 4)) break;
            if (u >= 0 && u < p.H) {
                uint8_t* vbuf = sVol + vb * p.vol_buf_bytes;
                if (FUSED && CORR >= 6) {
                    // CUDA-core correlation: the row's KG * n_fitems items
                    // (job-major) in tasks of 32; task tau of the row goes to
                    // warp (it * n_tasks + tau) mod kProdWarps.  A warp waits
                    // for every job up to the last one its next task touches
                    // and releases every job before that task's first one
                    // (a task spans at most fma_span <= n_slots jobs), and
                    // every warp waits for and releases all KG jobs in order.
                    const int job0 = (u - uv0) * p.KG;
                    const int P = 2 * p.n_fitems;  // (group half, table entry) items per job
                    const int n_items = p.KG * P;
                    const int n_tasks = (n_items + 31) / 32;
                    int waited = 0, released = 0;
                    for (int tau = ((pw - it * n_tasks) % kProdWarps + kProdWarps) % kProdWarps; tau < n_tasks && ok;
                         tau += kProdWarps) {
                        const int i0 = tau * 32;
                        const int kg_first = i0 / P, kg_last = (min(i0 + 32, n_items) - 1) / P;
                        for (; released < kg_first; ++released) {
                            __syncwarp();
                            if (lane == 0) mbar_arrive(smem_addr(&stage_empty[(job0 + released) % p.n_slots]));
                        }
                        for (; waited <= kg_last && ok; ++waited) {
                            const int job = job0 + waited;
                            ok = warp_wait(smem_addr(&stage_full[job % p.n_slots]), (job / p.n_slots) & 1, p.err, 7);
                        }
                        if (!ok) break;
                        const int item = i0 + lane;
                        if (item < n_items) {
                            const int kg = item / P;
                            const int job = job0 + kg;
                            const int k = item - kg * P;
                            const int q = k >= p.n_fitems ? 1 : 0;
                            corr_item<CORR>(p, smem + p.off_stage + (job % p.n_slots) * p.stage_slot_bytes,
                                            vbuf + kg * p.lbo_vol, k - q * p.n_fitems, q);
                        }
                    }
                    for (; waited < p.KG && ok; ++waited) {
                        const int job = job0 + waited;
                        ok = warp_wait(smem_addr(&stage_full[job % p.n_slots]), (job / p.n_slots) & 1, p.err, 7);
                    }
                    if (ok) {
                        __syncwarp();
                        for (; released < p.KG; ++released)
                            if (lane == 0) mbar_arrive(smem_addr(&stage_empty[(job0 + released) % p.n_slots]));
                    }
                } else if (FUSED) {
                    const int job0 = (u - uv0) * p.KG;  // job of (u, octet 0)
                    for (int kg = 0; kg < p.KG && ok; ++kg, next_job()) {
                        const int job = job0 + kg;
                        const int slot = js;
                        if (!warp_wait(smem_addr(&stage_full[slot]), jph, p.err, 7)) {
                            ok = false;
                            break;
                        }
                        const uint32_t sbase = smem_addr(smem + p.off_stage + slot * p.stage_slot_bytes);
                        const uint32_t vsa = smem_addr(vbuf + kg * p.lbo_vol);
                        // this warp's tasks of the job: tau = job * T + h with
                        // T = tpj * ntile tasks per job, tau % kProdWarps == pw;
                        // task h is range h % tpj of tile h / tpj.
                        const int T = p.tpj * NT;
                        static_assert((kProdWarps & (kProdWarps - 1)) == 0, "warp rotation by mask");
                        for (int h = (pw - job * T) & (kProdWarps - 1); h < T; h += kProdWarps) {
                            const int tl = (NT == 2 && h >= p.tpj) ? 1 : 0, hh = h - tl * p.tpj;
                            const int jt0 = p.task_jt[hh], jt1 = p.task_jt[hh + 1];
                            corr_task<CORR, NT>(p, sbase, zero_row, vsa + static_cast<uint32_t>(tl) * p.tile_vol_bytes,
                                                jt0, jt1, lane, tl);
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(smem_addr(&stage_empty[slot]));
                    }
                } else if (p.use_tma) {
                    // Volume mode, TMA-staged: job (u, octet kg) holds
                    // [8 groups][np planes][24 columns w0 - 8 .. w0 + 15]; one
                    // item per plane reads the 8 groups' interior columns as
                    // 16-byte rows (lanes 48 bytes apart: no bank conflicts)
                    // and the two halo columns, transposes in registers and
                    // writes the octet's rows w' = 0..9 of the plane.  Items
                    // of consecutive jobs start on different warps.
                    const int np = p.d_hi - p.d_lo;
                    const uint32_t gbytes = static_cast<uint32_t>(np) * 48u;
                    const int job0 = (u - uv0) * p.KG;
                    for (int kg = 0; kg < p.KG && ok; ++kg, next_job()) {
                        const int job = job0 + kg;
                        const int slot = js;
                        if (!warp_wait(smem_addr(&stage_full[slot]), jph, p.err, 7)) {
                            ok = false;
                            break;
                        }
                        const uint32_t sbase = smem_addr(smem + p.off_stage + slot * p.stage_slot_bytes);
                        const uint32_t vrow0 = smem_addr(vbuf + kg * p.lbo_vol);
                        int i = pw * 32 + lane - (job * np) % (kProdWarps * 32);
                        if (i < 0) i += kProdWarps * 32;
                        for (; i < np; i += kProdWarps * 32) {
                            const uint32_t src = sbase + static_cast<uint32_t>(i) * 48u;
                            uint32_t wg[8][4];
                            unsigned short h0[8], h9[8];
#pragma unroll
                            for (int g = 0; g < 8; ++g) {
                                ld_shared_v4(src + g * gbytes + 16u, wg[g]);
                                h0[g] = ld_shared_u16(src + g * gbytes + 14u);
                                h9[g] = ld_shared_u16(src + g * gbytes + 32u);
                            }
                            const uint32_t row = vrow0 + static_cast<uint32_t>((p.d_lo + i + 1) * kWtp * 16);
                            st_shared_v4(row, pack_b16x2(h0[0], h0[1]), pack_b16x2(h0[2], h0[3]),
                                         pack_b16x2(h0[4], h0[5]), pack_b16x2(h0[6], h0[7]));
                            st_shared_v4(row + 9 * 16, pack_b16x2(h9[0], h9[1]), pack_b16x2(h9[2], h9[3]),
                                         pack_b16x2(h9[4], h9[5]), pack_b16x2(h9[6], h9[7]));
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                st_shared_v4(row + (1 + 2 * k) * 16, __byte_perm(wg[0][k], wg[1][k], 0x5410),
                                             __byte_perm(wg[2][k], wg[3][k], 0x5410),
                                             __byte_perm(wg[4][k], wg[5][k], 0x5410),
                                             __byte_perm(wg[6][k], wg[7][k], 0x5410));
                                st_shared_v4(row + (2 + 2 * k) * 16, __byte_perm(wg[0][k], wg[1][k], 0x7632),
                                             __byte_perm(wg[2][k], wg[3][k], 0x7632),
                                             __byte_perm(wg[4][k], wg[5][k], 0x7632),
                                             __byte_perm(wg[6][k], wg[7][k], 0x7632));
                            }
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(smem_addr(&stage_empty[slot]));
                    }
                } else if (p.vec_ok) {
                    // Volume mode, 16-byte path (W % 8 == 0, aligned volume):
                    // one item per (octet, plane d) -- the 8 groups' interior
                    // columns w0 .. w0 + 7 as one 16-byte load each, an 8 x 8
                    // transpose in registers, and the two halo columns -- so
                    // the octet's rows w' = 0..9 of plane d are written as ten
                    // 16-byte rows.
                    const int64_t plane = i64(p.H) * p.W;
                    const int64_t gstride = i64(p.D_tot) * plane;
                    const int nd = p.d_hi - p.d_lo;
                    for (int i = pw * 32 + lane; i < p.KG * nd; i += kProdWarps * 32) {
                        const int kg = i / nd;
                        const int d = p.d_lo + (i - kg * nd);  // band-relative; plane d + 1
                        const __half* src =
                            p.vol + ((i64(b) * p.G + 8 * kg) * p.D_tot + p.d_off + d) * plane + i64(u) * p.W + w0;
                        uint4 r[8];
                        unsigned short h0[8], h9[8];
#pragma unroll
                        for (int g = 0; g < 8; ++g) {
                            r[g] = make_uint4(0u, 0u, 0u, 0u);
                            h0[g] = 0;
                            h9[g] = 0;
                            if (8 * kg + g < p.G) {
                                const __half* s = src + g * gstride;
                                r[g] = __ldg(reinterpret_cast<const uint4*>(s));
                                if (w0 > 0) h0[g] = __half_as_ushort(__ldg(s - 1));
                                if (w0 + 8 < p.W) h9[g] = __half_as_ushort(__ldg(s + 8));
                            }
                        }
                        const uint32_t row = smem_addr(vbuf + kg * p.lbo_vol + (d + 1) * kWtp * 16);
                        st_shared_v4(row, pack_b16x2(h0[0], h0[1]), pack_b16x2(h0[2], h0[3]), pack_b16x2(h0[4], h0[5]),
                                     pack_b16x2(h0[6], h0[7]));
                        st_shared_v4(row + 9 * 16, pack_b16x2(h9[0], h9[1]), pack_b16x2(h9[2], h9[3]),
                                     pack_b16x2(h9[4], h9[5]), pack_b16x2(h9[6], h9[7]));
                        // Column j of the interior is half j of every group's
                        // load: word k of group g holds columns 2k, 2k + 1.
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            uint32_t wg[8];
#pragma unroll
                            for (int g = 0; g < 8; ++g)
                                wg[g] = k == 0 ? r[g].x : (k == 1 ? r[g].y : (k == 2 ? r[g].z : r[g].w));
                            st_shared_v4(row + (1 + 2 * k) * 16, __byte_perm(wg[0], wg[1], 0x5410),
                                         __byte_perm(wg[2], wg[3], 0x5410), __byte_perm(wg[4], wg[5], 0x5410),
                                         __byte_perm(wg[6], wg[7], 0x5410));
                            st_shared_v4(row + (2 + 2 * k) * 16, __byte_perm(wg[0], wg[1], 0x7632),
                                         __byte_perm(wg[2], wg[3], 0x7632), __byte_perm(wg[4], wg[5], 0x7632),
                                         __byte_perm(wg[6], wg[7], 0x7632));
                        }
                    }
                } else {
                    for (int kg = 0; kg < p.KG; ++kg) {
                        // Volume mode: gather vol[b, g, d, u, w] into the octet's rows.
                        const int64_t plane = i64(p.H) * p.W;
                        for (int i = pw * 32 + lane; i < 8 * (p.d_hi - p.d_lo) * kWtp; i += kProdWarps * 32) {
                            const int ge = i % 8;
                            const int rest = i / 8;
                            const int wp = rest % kWtp;
                            const int d = p.d_lo + rest / kWtp;  // band-relative; plane d + 1
                            const int g = kg * 8 + ge;
                            const int wa = w0 - 1 + wp;
                            __half v = __float2half_rn(0.0f);
                            if (g < p.G && wa >= 0 && wa < p.W)
                                v = p.vol[((i64(b) * p.G + g) * p.D_tot + p.d_off + d) * plane + i64(u) * p.W + wa];
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

// CTAs of `kernel` resident per SM with `smem` bytes of dynamic shared
// memory (registers, threads and shared memory; 0 = a CUDA call failed).
// The first call for a (kernel, device) raises the kernel's dynamic
// shared-memory limit to the device's opt-in maximum, so launches with any
// smaller size need nothing more; both driver queries are cached per
// (kernel, device, smem) instead of running on every launch.
int resident_ctas(const void* kernel, int device, int optin, size_t smem) noexcept
{
    constexpr int kSlots = 64;
    struct Entry { const void* fn; int dev; size_t smem; int ctas; };
    static std::mutex mu;
    static Entry done[kSlots];
    static int n_done = 0;
    std::lock_guard<std::mutex> lock(mu);
    bool raised = false;
    for (int i = 0; i < n_done; ++i) {
        if (done[i].fn != kernel || done[i].dev != device) continue;
        raised = true;
        if (done[i].smem == smem) return done[i].ctas;
    }
    if (!raised && cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin) != cudaSuccess)
        return 0;
    int ctas = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&ctas, kernel, kThreads, smem) != cudaSuccess || ctas < 1)
        return 0;
    if (n_done < kSlots) done[n_done++] = Entry{kernel, device, smem, ctas};
    return ctas;
}

uint32_t pow2_cols(uint32_t c)
{
    uint32_t r = 32;
    while (r < c) r <<= 1;
    return r;
}

}  // namespace

int corr_scale_div_grouped(bool is_half, int B, int C, int G, int H, int W, int D, int sm_count) noexcept;

int set_fused_corr_engine(int engine) noexcept
{
    if (engine != WW_CORR_ENGINE_TENSOR && engine != WW_CORR_ENGINE_CUDA_CORES) return WW_ERR_INVALID_SHAPE;
    return g_corr_engine.exchange(engine);
}

int fused_corr_engine() noexcept
{
    return g_corr_engine.load();
}

// The two-tile instantiation of a fused variant (Cout <= 16 and the
// tensor-core correlation variants only; nullptr for the others).
template <int CP, int CV>
constexpr void (*dual_tile_kernel())(StemParams)
{
    if constexpr (CP == 16 && CV >= 1 && CV <= 4) return stem_tc_kernel<CP, true, CV, 2>;
    else return nullptr;
}

namespace {

// Whether one launch takes a band of Db disparities (halo: the band has a
// volume plane above it, which widens the staged right window by one
// disparity): the stem's accumulators -- three Cout-column slots per
// 16-disparity M-block -- within the 512 tensor-memory columns, at most
// kMaxSteps K-steps (G <= 56), and the smallest shared-memory layout -- B
// image, two volume-row buffers, two staging slots -- within smem_optin.
bool band_fits(bool fused, int C, int G, int Db, int Cout, int smem_optin, bool halo) noexcept
{
    const int coutp = Cout <= 16 ? 16 : 32;
    const int KG = (G + 7) / 8;
    const int Dp = (Db + 15) / 16 * 16;
    const int n_mb = Dp / 16;
    if (n_mb * 3 * coutp > 512 || n_mb > kMaxMB) return false;
    const int nsteps = 9 * (KG / 2) + ((KG & 1) ? 5 : 0);
    if (nsteps > kMaxSteps) return false;
    const long long Cg = fused ? C / G : 1;
    const long long vol_buf = static_cast<long long>(Dp + 2) * kWtp * 16 * KG + 128;
    long long o = static_cast<long long>(nsteps) * 2 * 5 * coutp * 16;
    o = (o + 127) & ~127LL;
    o += 2 * vol_buf;
    o = (o + 127) & ~127LL;
    o += 128 + (2 * kMaxVBuf + 1 + 2 * kMaxSlots + 4) * 8 + 16;
    o = (o + 15) & ~15LL;
    o += coutp * 4;
    o = (o + 1023) & ~1023LL;
    if (fused) {
        const long long rstage_w = 16 + 8 * ((Db + (halo ? 1 : 0) + 7) / 8);
        const long long n_rbox = (rstage_w + 63) / 64;
        const long long slot = ((n_rbox * 8 * Cg * 128 + 8 * Cg * kLRowBytes + 1023) / 1024) * 1024;
        o += 2 * slot;
    }
    return o <= smem_optin;
}

// Disparities per launch for a D-disparity volume: D when one launch takes
// it, else the largest multiple of 16 that a band (with its halo planes)
// fits; 0 when not even a 16-disparity band fits.
int max_band(bool fused, int C, int G, int D, int Cout, int smem_optin) noexcept
{
    if (band_fits(fused, C, G, D, Cout, smem_optin, false)) return D;
    for (int Db = (D - 1) / 16 * 16; Db >= 16; Db -= 16)
        if (band_fits(fused, C, G, Db, Cout, smem_optin, true)) return Db;
    return 0;
}

}  // namespace

// Whether the stem kernel takes a shape: WW_SUCCESS, WW_ERR_INVALID_SHAPE or
// WW_ERR_UNSUPPORTED.  The limits of this build: Cout <= 32; G <= 56 (at
// most kMaxSteps K-steps); and a band of 16 disparities (or all of them when
// fewer) must fit shared memory -- B image, two volume-row buffers, two
// staging slots -- which bounds G further.  Any D is taken: disparity ranges
// that one launch cannot hold run as several bands (stem_tc_launch).
// fused: the correlation feeds the stem (C channels in G groups); otherwise a
// G-channel volume is read.
int stem_limits(bool fused, int C, int G, int D, int Cout, int smem_optin) noexcept
{
    if (C <= 0 || G <= 0 || D <= 0 || Cout <= 0) return WW_ERR_INVALID_SHAPE;
    if (fused && C % G != 0) return WW_ERR_INVALID_SHAPE;
    if (Cout > 32) return WW_ERR_UNSUPPORTED;
    return max_band(fused, C, G, D, Cout, smem_optin) > 0 ? WW_SUCCESS : WW_ERR_UNSUPPORTED;
}

namespace {

// One launch over disparities [d_off, d_off + D) of a D_tot-disparity volume.
int stem_tc_launch_band(const void* vol, const void* left, const void* right, const void* w, const void* b,
                        void* out, int B, int C, int G, int H, int W, int D_tot, int d_off, int D, int Cout, int act,
                        int in_row0, int in_rows, int out_row0, int out_rows, cudaStream_t stream,
                        const DeviceInfo& dev) noexcept
{
    const bool fused = (vol == nullptr);

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
    p.d_off = d_off;
    p.D_tot = D_tot;
    p.d_lo = d_off > 0 ? -1 : 0;                // the plane below the band: real data, or the zero padding
    p.d_hi = d_off + D < D_tot ? D + 1 : D;     // the plane above the band likewise
    p.n8 = (p.d_hi + 7) / 8;
    p.in_row0 = in_row0; p.in_rows = in_rows; p.out_row0 = out_row0; p.out_rows = out_rows;
    p.Cg = Cg; p.KG = KG; p.Dp = Dp; p.n_mb = n_mb; p.nsteps = nsteps;
    // The fused correlation scales by * (1 / Cg): exactly / Cg when Cg is a
    // power of two, within one fp32 ulp of it otherwise (the tensor-core sums
    // already differ from CorrVolume's fp32 chain at that level), and without
    // a division subroutine per value.
    p.inv_cg = 1.0f / static_cast<float>(Cg);
    // 16-byte loads: the features (fused) or the volume (volume mode).
    p.vec_ok = (W % 8 == 0) && (fused ? (reinterpret_cast<uintptr_t>(left) % 16 == 0 &&
                                         reinterpret_cast<uintptr_t>(right) % 16 == 0)
                                      : reinterpret_cast<uintptr_t>(vol) % 16 == 0);
    const bool cuda_core_corr = fused && g_corr_engine.load(std::memory_order_relaxed) == WW_CORR_ENGINE_CUDA_CORES;
    // Volume mode stages [8 groups][planes][24 columns] boxes by TMA when the
    // volume allows 16-byte rows (else the producers gather it themselves).
    const int n_planes = p.d_hi - p.d_lo;
    bool vol_tma = !fused && p.vec_ok && n_planes <= 256;

    // Geometry for nt 8-column tiles per CTA; returns the dynamic shared
    // memory, or 0 when it does not fit (or, for two tiles, leaves fewer
    // than three staging slots).  Shared-memory layout: B image | 2 or 3
    // volume buffers (each nt tiles) | zero row, barriers, bias | staging ring
    // (1024-byte aligned slots for the 128-byte TMA swizzle).  Three volume
    // buffers when three staging slots still fit.
    auto geometry = [&](int nt) -> size_t {
        p.ntile = nt;
        p.l_stage_w = lstage_w(nt);
        p.l_row_bytes = 2 * p.l_stage_w;
        p.n_wtiles = (W + kWt * nt - 1) / (kWt * nt);
        p.rstage_w = 16 + 8 * p.n8 + kWt * (nt - 1);  // right columns [w0 - d_off - 8 n8, w0 - d_off + 8 nt + 8)
        p.tmem_cols = pow2_cols(static_cast<uint32_t>(nt * n_mb * 3 * coutp));
        p.lbo_vol = static_cast<uint32_t>((Dp + 2) * kWtp * 16);
        // + a zeroed 128-byte guard per tile: the zero-weight partner of a lone
        // octet (step_info, t1 < 0) reads one 16-byte position past the last plane.
        p.tile_vol_bytes = p.lbo_vol * KG + 128;
        p.vol_buf_bytes = static_cast<uint32_t>(nt) * p.tile_vol_bytes;
        p.n_tiles = p.n8 + 2;
        p.n_rbox = (p.rstage_w + 63) / 64;
        p.rbox_bytes = static_cast<uint32_t>(8 * Cg * 128);
        p.off_l = static_cast<uint32_t>(p.n_rbox) * p.rbox_bytes;
        p.stage_slot_bytes =
            fused ? ((p.off_l + 8u * Cg * static_cast<uint32_t>(p.l_row_bytes) + 1023) / 1024) * 1024
                  : (vol_tma ? ((8u * 48u * static_cast<uint32_t>(n_planes) + 127) / 128) * 128 : 0);
        p.stage_tx = fused ? static_cast<uint32_t>((p.n_rbox * 64 + p.l_stage_w) * 8 * Cg * 2)
                           : 8u * 48u * static_cast<uint32_t>(n_planes);
        auto bar_bytes = [&](int ns) { return static_cast<uint32_t>((2 * kMaxVBuf + 1 + 2 * ns + 4) * 8 + 16); };
        auto layout = [&](int nv) -> uint32_t {  // offset of the staging ring for nv volume buffers
            uint32_t o = static_cast<uint32_t>(nsteps) * 2 * 5 * coutp * 16;
            o = (o + 127) & ~127u;
            p.off_vol = o;
            o += static_cast<uint32_t>(nv) * p.vol_buf_bytes;
            o = (o + 127) & ~127u;
            p.off_zero = o;
            o += 128;
            p.off_bar = o;
            o += bar_bytes(kMaxSlots);
            o = (o + 15) & ~15u;
            p.off_bias = o;
            o += static_cast<uint32_t>(coutp) * 4;
            return (o + 1023) & ~1023u;
        };
        p.n_vbuf = (layout(3) + 3 * p.stage_slot_bytes <= static_cast<uint32_t>(dev.smem_optin)) ? 3 : 2;
        uint32_t off = layout(p.n_vbuf);
        p.off_b = 0;
        p.off_stage = off;
        // as many staging slots (2..kMaxSlots) as shared memory holds
        p.n_slots = 2;
        const bool staged = fused || vol_tma;
        while (staged && p.n_slots < kMaxSlots &&
               off + (p.n_slots + 1) * p.stage_slot_bytes <= static_cast<uint32_t>(dev.smem_optin))
            ++p.n_slots;
        off += staged ? p.n_slots * p.stage_slot_bytes : 0;
        if (off > static_cast<uint32_t>(dev.smem_optin)) return 0;
        if (nt == 2 && p.n_slots < 3) return 0;
        return off;
    };
    // Two column tiles per CTA when their accumulators fit tensor memory
    // (Cout <= 16, D <= 80) and the tensor-core correlation runs: the right
    // window staged per job then serves 16 output columns instead of 8, and
    // one tile's drain overlaps the other's MMAs.
    size_t smem = 0;
    if (fused && kDualTiles && !cuda_core_corr && coutp == 16 && Cg <= 16 && W > kWt &&
        2 * n_mb * 3 * coutp <= 512)
        smem = geometry(2);
    if (smem == 0) smem = geometry(1);
    if (vol_tma && (smem == 0 || !encode_volume_map(&p.tmap_l, vol, B, G, D_tot, H, W, 24, n_planes, 8))) {
        vol_tma = false;  // no room for the staging ring (or no map): the producers gather
        smem = geometry(1);
    }
    if (smem == 0) return WW_ERR_UNSUPPORTED;
    // M-block groups: one per tile with two tiles; otherwise two from
    // kGroupMinMB M-blocks on (each group keeps at least two M-blocks
    // interleaved, so its MMAs stay independent).
    p.n_grp = p.ntile == 2 ? 2 : (n_mb >= kGroupMinMB ? 2 : 1);
    p.grp_size = p.ntile == 2 ? n_mb : (n_mb + p.n_grp - 1) / p.n_grp;
    // Tasks per job: two right tiles per task with one column tile per CTA,
    // four with two.  A task loads its octet's left (A) fragments once for all
    // its tiles, so more tiles per task mean fewer of those loads, while
    // enough producer warps per job keep a job's latency (and so the staging
    // ring's turnover) short.  Measured: two tiles 7 % faster than one on
    // config 2, three and four tiles slower on configs 2 and 4 (3 % and 5 %
    // with four); with two column tiles (twice the tasks per job) four tiles
    // per task are 2.5 % faster on config 3 and equal on config 5.
    const int tiles_per_task = p.ntile == 2 ? 4 : 2;
    p.tpj = (p.n_tiles + tiles_per_task - 1) / tiles_per_task;
    if (p.tpj > kMaxTasks) return WW_ERR_UNSUPPORTED;
    for (int hh = 0; hh <= p.tpj; ++hh) p.task_jt[hh] = static_cast<uint8_t>((hh * p.n_tiles) / p.tpj);
    // CUDA-core correlation items: (right tile, volume column) pairs with
    // any disparity in [0, D), and the most jobs a task of 32 items touches.
    p.n_fitems = 0;
    p.fma_span = 0;
    p.scale_div = 0;
    if (cuda_core_corr) {
        // (* 1 / Cg is exactly / Cg when Cg is a power of two)
        p.scale_div = (Cg & (Cg - 1)) == 0 ? 0 : corr_scale_div_grouped(true, B, C, G, H, W, D, dev.sm_count);
        const int dbase = 8 * (p.n_tiles - 2) - 1;
        for (int jt = 0; jt < p.n_tiles; ++jt)
            for (int wp = 0; wp < kWtp; ++wp) {
                const int dmax = dbase + wp - 8 * jt, dmin = dmax - 7;
                if (dmax < p.d_lo || dmin > p.d_hi - 1) continue;
                if (p.n_fitems >= kMaxFItems) return WW_ERR_UNSUPPORTED;
                const bool full = dmin >= p.d_lo && dmax <= p.d_hi - 1;
                p.fitems[p.n_fitems++] = static_cast<uint16_t>(wp | (jt << 4) | (full ? 0x8000 : 0));
            }
        const int per_job = 2 * p.n_fitems;  // two group halves per entry
        const int n_items = KG * per_job;
        for (int i0 = 0; i0 < n_items; i0 += 32)
            p.fma_span = std::max(p.fma_span, (std::min(i0 + 32, n_items) - 1) / per_job - i0 / per_job + 1);
        if (p.fma_span > p.n_slots) return WW_ERR_UNSUPPORTED;
    }
    p.out_vec = (W % 8 == 0) && (reinterpret_cast<uintptr_t>(out) % 16 == 0);
    {
        const size_t wbytes = static_cast<size_t>(Cout) * G * 54;
        const bool fits = wbytes <= static_cast<size_t>(p.n_vbuf) * p.vol_buf_bytes;
        p.raw_w_smem = !fits ? 0
                       : (G % 8 == 0) ? 2
                       : ((reinterpret_cast<uintptr_t>(w) % 16 == 0) && (wbytes % 16 == 0)) ? 1 : 0;
    }
    p.use_tma = vol_tma ? 1 : 0;
    if (fused && p.vec_ok && 8 * Cg <= 256) {
        p.use_tma = encode_feature_map(&p.tmap_l, left, B, C, in_rows, W, p.l_stage_w, 8 * Cg, false) &&
                    encode_feature_map(&p.tmap_r, right, B, C, in_rows, W, 64, 8 * Cg, true);
    }

    // Descriptor templates (base address 0; the kernel adds its buffer bases)
    // and the B image's per-chunk weight offsets.
    for (int s = 0; s < nsteps; ++s) {
        const StepInfo si = step_info(s, KG);
        for (int c = 0; c < 2; ++c) {
            const int tap = c ? si.t1 : si.t0, kg = c ? si.kg1 : si.kg0;
            p.step_off[2 * s + c] = tap < 0 ? -1 : 8 * kg * 27 + (tap / 3) * 9 + (tap % 3);
            p.step_gv[2 * s + c] = std::min(8, G - 8 * kg);
        }
        const uint32_t off0 = si.kg0 * p.lbo_vol + tap_shift(si.t0);
        const uint32_t off1 = si.t1 >= 0 ? si.kg1 * p.lbo_vol + tap_shift(si.t1) : off0 + 16;
        p.tmplA[s] = host_smem_desc(off0, off1 - off0, kWtp * 16);
        p.tmplB[s] = host_smem_desc(static_cast<uint32_t>(s * 2 * 5 * coutp * 16), 5 * coutp * 16, 128);
    }

    using KernelFn = void (*)(StemParams);
    KernelFn kernel = nullptr;
    if (!fused) {
        kernel = coutp == 16 ? stem_tc_kernel<16, false, 0, 1> : stem_tc_kernel<32, false, 0, 1>;
    } else {
        const int cv = corr_variant(Cg, cuda_core_corr);
#define WW_FUSED_CASE(CP, CV) \
    if (coutp == CP && cv == CV) kernel = p.ntile == 2 ? dual_tile_kernel<CP, CV>() : stem_tc_kernel<CP, true, CV, 1>;
        WW_FUSED_CASE(16, 1) WW_FUSED_CASE(16, 2) WW_FUSED_CASE(16, 3) WW_FUSED_CASE(16, 4) WW_FUSED_CASE(16, 5)
        WW_FUSED_CASE(32, 1) WW_FUSED_CASE(32, 2) WW_FUSED_CASE(32, 3) WW_FUSED_CASE(32, 4) WW_FUSED_CASE(32, 5)
        WW_FUSED_CASE(16, 6) WW_FUSED_CASE(16, 7) WW_FUSED_CASE(16, 8) WW_FUSED_CASE(16, 9) WW_FUSED_CASE(16, 10)
        WW_FUSED_CASE(32, 6) WW_FUSED_CASE(32, 7) WW_FUSED_CASE(32, 8) WW_FUSED_CASE(32, 9) WW_FUSED_CASE(32, 10)
#undef WW_FUSED_CASE
    }
    if (kernel == nullptr) return WW_ERR_UNSUPPORTED;
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return WW_ERR_DEVICE;
    const char* op = fused ? "ww_corr_cost_stem3d" : "ww_cost_stem3d";
    const int resident = resident_ctas(reinterpret_cast<const void*>(kernel), device, dev.smem_optin, smem);
    if (resident == 0) return launch_status(op);

    // Strip length: minimise (waves of CTAs) x (rows streamed per CTA), with
    // the CTAs an SM holds at once limited by registers, shared memory and
    // the tensor-memory columns each CTA allocates (at 448 threads and
    // 120-128 registers a thread the fused kernel runs one CTA per SM).
    const long long col_tiles = static_cast<long long>(B) * p.n_wtiles;
    const int ctas_per_sm = std::max(1, std::min(resident, static_cast<int>(512 / p.tmem_cols)));
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
    kernel<<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(p);
    return launch_status(op);
}

}  // namespace

// Disparity bands: when the whole range does not fit one launch (tensor
// memory holds three Cout-column accumulators per 16 disparities; shared
// memory the weights, volume rows and staging), the volume is computed in
// bands of the largest multiple of 16 disparities that fits, one launch each.
// A band's volume buffer also holds the plane below and above it (real
// correlation values, or the conv's zero padding at the ends), so every
// output value sees exactly the taps it sees in one launch.
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
    const int band = max_band(fused, C, G, D, Cout, dev.smem_optin);
    if (band <= 0) return stem_limits(fused, C, G, D, Cout, dev.smem_optin);
    for (int d0 = 0; d0 < D; d0 += band) {
        const int st = stem_tc_launch_band(vol, left, right, w, b, out, B, C, G, H, W, D, d0, std::min(band, D - d0),
                                           Cout, act, in_row0, in_rows, out_row0, out_rows, stream, dev);
        if (st != WW_SUCCESS) return st;
    }
    return WW_SUCCESS;
}

}  // namespace ww

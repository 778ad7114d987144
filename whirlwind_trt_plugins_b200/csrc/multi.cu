// multi.cu -- host driver that runs the fused CorrVolume -> CostStem3D op
// (ww_corr_cost_stem3d) over several devices from one host thread.
//
//   WW_MULTI_BATCH  part k computes batch items split_even(B, n, k) on its
//                   device; nothing moves between devices.
//   WW_MULTI_ROWS   one image pair split into row bands: part k owns image
//                   rows [r0, r1) = split_even(H, n, k) and holds them in a
//                   band buffer of rows [i0, i1) (one halo row each side,
//                   clipped to the image).  The halo rows are the
//                   neighbours' first / last own rows: one strided peer copy
//                   each (cudaMemcpy3DPeerAsync, over NVLink between GPUs)
//                   on the part's stream, ordered after the neighbour's
//                   stream by an event; then the band form of the kernel
//                   runs on the part's rows.  Correlation is row-local and
//                   the stem reaches one row up and down, so the stitched
//                   output equals the single-device call bit for bit.
// No collective runs inside the op and no kernel reads another device's
// memory: remote rows are copied into the part's own buffer first.
// Several parts may name the same device (their copies are then
// device-local), which lets one GPU run the row-band path.
#include "ww_common.cuh"

#include <atomic>
#include <mutex>

namespace ww {

namespace {

constexpr int kMaxParts = 64;

// Test hook (ww_multi_inject_copy_failure): number of halo copies still
// issued before one is made to fail; negative = no injection.
std::atomic<int> g_copy_fail_after{-1};

void split_even(int n, int world, int k, int* s, int* e)
{
    const int base = n / world, extra = n % world;
    *s = k * base + (k < extra ? k : extra);
    *e = *s + base + (k < extra ? 1 : 0);
}

// Peer access between two distinct devices, enabled once per ordered pair
// (a direct NVLink path for the halo copies; without it the runtime stages
// the copy, which is slower but correct).
void ensure_peer_access(int dev, int peer) noexcept
{
    if (dev == peer) return;
    static std::mutex mu;
    static bool done[kMaxParts][kMaxParts];
    if (dev < 0 || peer < 0 || dev >= kMaxParts || peer >= kMaxParts) return;
    std::lock_guard<std::mutex> lock(mu);
    if (done[dev][peer]) return;
    done[dev][peer] = true;
    int can = 0;
    if (cudaDeviceCanAccessPeer(&can, dev, peer) != cudaSuccess || !can) {
        cudaGetLastError();
        return;
    }
    int cur = 0;
    cudaGetDevice(&cur);
    if (cudaSetDevice(dev) == cudaSuccess) {
        const cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
        if (e != cudaSuccess) cudaGetLastError();  // e.g. already enabled
    }
    cudaSetDevice(cur);
}

// Copy image row `src_row` of a [B*C][src_rows][W] fp16 band (device
// src_dev) into row `dst_row` of a [B*C][dst_rows][W] band (device dst_dev):
// B*C rows of W*2 bytes, one strided copy.
cudaError_t copy_row(void* dst, int dst_dev, int dst_rows, int dst_row, const void* src, int src_dev, int src_rows,
                     int src_row, int BC, int W, cudaStream_t stream) noexcept
{
    int left = g_copy_fail_after.load();
    while (left >= 0) {
        if (left == 0) {
            if (g_copy_fail_after.compare_exchange_strong(left, -1)) return cudaErrorInvalidValue;
            continue;
        }
        if (g_copy_fail_after.compare_exchange_strong(left, left - 1)) break;
    }
    const size_t rb = static_cast<size_t>(W) * 2;
    cudaMemcpy3DPeerParms q{};
    q.srcPtr = make_cudaPitchedPtr(const_cast<void*>(src), rb, rb, static_cast<size_t>(src_rows));
    q.srcPos = make_cudaPos(0, static_cast<size_t>(src_row), 0);
    q.srcDevice = src_dev;
    q.dstPtr = make_cudaPitchedPtr(dst, rb, rb, static_cast<size_t>(dst_rows));
    q.dstPos = make_cudaPos(0, static_cast<size_t>(dst_row), 0);
    q.dstDevice = dst_dev;
    q.extent = make_cudaExtent(rb, 1, static_cast<size_t>(BC));
    return cudaMemcpy3DPeerAsync(&q, stream);
}

struct DeviceRestore {
    int dev = -1;
    DeviceRestore() { if (cudaGetDevice(&dev) != cudaSuccess) dev = -1; }
    ~DeviceRestore() { if (dev >= 0) cudaSetDevice(dev); }
};

int fail(cudaError_t e) noexcept
{
    std::fprintf(stderr, "[ww_trt_plugins] ww_corr_cost_stem3d_multi: CUDA call failed: %s\n", cudaGetErrorString(e));
    cudaGetLastError();
    return WW_ERR_LAUNCH;
}

}  // namespace

}  // namespace ww

extern "C" {

int ww_multi_split(int n, int H, int k, int* r0, int* r1, int* i0, int* i1)
{
    if (r0 == nullptr || r1 == nullptr || i0 == nullptr || i1 == nullptr) return WW_ERR_NULL_POINTER;
    if (n <= 0 || n > ww::kMaxParts || k < 0 || k >= n || H < n) return WW_ERR_INVALID_SHAPE;
    ww::split_even(H, n, k, r0, r1);
    *i0 = *r0 > 0 ? *r0 - 1 : 0;
    *i1 = *r1 < H ? *r1 + 1 : H;
    return WW_SUCCESS;
}

int ww_multi_inject_copy_failure(int after_n_copies)
{
    ww::g_copy_fail_after.store(after_n_copies < 0 ? -1 : after_n_copies);
    return WW_SUCCESS;
}

int ww_corr_cost_stem3d_multi(int n, const int* devices, int mode, void* const* left, void* const* right,
                              const void* const* w, const void* const* b, void* const* out, int B, int C, int G,
                              int H, int W, int D, int Cout, int act, void* const* streams)
{
    using namespace ww;
    // ---- argument checks (no CUDA call before they pass) ----
    if (devices == nullptr || left == nullptr || right == nullptr || w == nullptr || b == nullptr || out == nullptr)
        return WW_ERR_NULL_POINTER;
    if (n <= 0 || n > kMaxParts) return WW_ERR_INVALID_SHAPE;
    if (mode != WW_MULTI_BATCH && mode != WW_MULTI_ROWS) return WW_ERR_INVALID_SHAPE;
    if (B < 0 || C <= 0 || G <= 0 || H < 0 || W < 0 || D < 0 || Cout <= 0 || C % G != 0) return WW_ERR_INVALID_SHAPE;
    if (mode == WW_MULTI_ROWS && H < n) return WW_ERR_INVALID_SHAPE;
    for (int k = 0; k < n; ++k) {
        if (devices[k] < 0) return WW_ERR_INVALID_SHAPE;
        if (left[k] == nullptr || right[k] == nullptr || w[k] == nullptr || b[k] == nullptr || out[k] == nullptr)
            return WW_ERR_NULL_POINTER;
    }
    if (B == 0 || W == 0 || D == 0 || H == 0) return WW_SUCCESS;
    auto stream_of = [&](int k) {
        return streams != nullptr ? static_cast<cudaStream_t>(streams[k]) : static_cast<cudaStream_t>(nullptr);
    };
    DeviceRestore restore;

    if (mode == WW_MULTI_BATCH) {
        for (int k = 0; k < n; ++k) {
            int b0 = 0, b1 = 0;
            split_even(B, n, k, &b0, &b1);
            if (b1 == b0) continue;
            cudaError_t e = cudaSetDevice(devices[k]);
            if (e != cudaSuccess) return fail(e);
            const int st = ww_corr_cost_stem3d(left[k], right[k], w[k], b[k], out[k], b1 - b0, C, G, H, W, D, Cout,
                                               act, stream_of(k));
            if (st != WW_SUCCESS) return st;
        }
        return WW_SUCCESS;
    }

    // ---- row bands ----
    int r0[kMaxParts], r1[kMaxParts], i0[kMaxParts], i1[kMaxParts];
    for (int k = 0; k < n; ++k) ww_multi_split(n, H, k, &r0[k], &r1[k], &i0[k], &i1[k]);
    for (int k = 0; k + 1 < n; ++k) {
        ensure_peer_access(devices[k], devices[k + 1]);
        ensure_peer_access(devices[k + 1], devices[k]);
    }
    // ready[k]: everything enqueued on part k's stream so far (its own rows
    // written); copied[k]: part k's halo copies done (its neighbours' own
    // rows may then be overwritten by work enqueued after this call).
    cudaEvent_t ready[kMaxParts] = {}, copied[kMaxParts] = {};
    int status = WW_SUCCESS;
    auto cleanup = [&]() {
        for (int k = 0; k < n; ++k) {
            if (ready[k] != nullptr || copied[k] != nullptr) cudaSetDevice(devices[k]);
            if (ready[k] != nullptr) cudaEventDestroy(ready[k]);  // deferred until it completes
            if (copied[k] != nullptr) cudaEventDestroy(copied[k]);
        }
    };
    for (int k = 0; k < n && status == WW_SUCCESS; ++k) {
        cudaError_t e = cudaSetDevice(devices[k]);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ready[k], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&copied[k], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventRecord(ready[k], stream_of(k));
        if (e != cudaSuccess) status = fail(e);
    }
    const int BC = B * C;
    for (int k = 0; k < n && status == WW_SUCCESS; ++k) {
        cudaError_t e = cudaSetDevice(devices[k]);
        const cudaStream_t s = stream_of(k);
        const int rows = i1[k] - i0[k];
        if (e == cudaSuccess && k > 0) e = cudaStreamWaitEvent(s, ready[k - 1], 0);
        if (e == cudaSuccess && k + 1 < n) e = cudaStreamWaitEvent(s, ready[k + 1], 0);
        for (int t = 0; t < 2 && e == cudaSuccess; ++t) {
            void* dst = t == 0 ? left[k] : right[k];
            if (k > 0) {  // row r0 - 1: the last own row of part k - 1
                const void* src = t == 0 ? left[k - 1] : right[k - 1];
                e = copy_row(dst, devices[k], rows, 0, src, devices[k - 1], i1[k - 1] - i0[k - 1],
                             r1[k - 1] - 1 - i0[k - 1], BC, W, s);
            }
            if (e == cudaSuccess && k + 1 < n) {  // row r1: the first own row of part k + 1
                const void* src = t == 0 ? left[k + 1] : right[k + 1];
                e = copy_row(dst, devices[k], rows, rows - 1, src, devices[k + 1], i1[k + 1] - i0[k + 1],
                             r0[k + 1] - i0[k + 1], BC, W, s);
            }
        }
        if (e == cudaSuccess) e = cudaEventRecord(copied[k], s);
        if (e != cudaSuccess) {
            status = fail(e);
            break;
        }
        const int st = ww_corr_cost_stem3d_band(left[k], right[k], w[k], b[k], out[k], B, C, G, H, W, D, Cout, act,
                                                i0[k], rows, r0[k], r1[k] - r0[k], s);
        if (st != WW_SUCCESS) status = st;
    }
    // Work enqueued later on a neighbour's stream (new rows for the next
    // frame) waits for this call's copies out of its rows.
    for (int k = 0; k < n && status == WW_SUCCESS; ++k) {
        cudaError_t e = cudaSetDevice(devices[k]);
        if (e == cudaSuccess && k > 0) e = cudaStreamWaitEvent(stream_of(k), copied[k - 1], 0);
        if (e == cudaSuccess && k + 1 < n) e = cudaStreamWaitEvent(stream_of(k), copied[k + 1], 0);
        if (e != cudaSuccess) status = fail(e);
    }
    cleanup();
    return status;
}

}  // extern "C"

// tensor_map.cuh -- host-side encoding of TMA tensor maps for the NCHW fp16
// feature maps, through the driver entry point fetched from the runtime (no
// link-time dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace ww {

// 4-D tiled map over a contiguous [B, C, rows, W] fp16 tensor: dimensions
// (x = W, y = row, z = channel, w = batch), box (box_x, 1, box_z, 1).
// swizzle128: 128-byte swizzle of the box rows (box_x * 2 must be <= 128).
// Returns false when the shape cannot be described (W % 8 != 0, base not
// 16-byte aligned, box larger than 256 in a dimension) or encoding fails.
bool encode_feature_map(CUtensorMap* out, const void* base, int B, int C, int rows, int W, int box_x, int box_z,
                        bool swizzle128) noexcept;

// 5-D tiled map over a contiguous [B, G, D, H, W] fp16 volume: dimensions
// (x = W, y = row, z = disparity plane, g = group, b = batch), box
// (box_x, 1, box_d, box_g, 1), no swizzle.  Same conditions as above.
bool encode_volume_map(CUtensorMap* out, const void* base, int B, int G, int D, int H, int W, int box_x, int box_d,
                       int box_g) noexcept;

}  // namespace ww

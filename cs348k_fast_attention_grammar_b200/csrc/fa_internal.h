// Host-side helpers shared by the .cu files of the library (not part of the
// public C ABI, which is include/fa_b200.h).
#pragma once

#include <atomic>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/fa_b200.h"

namespace fa {

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library needs no link-time dependency on libcuda.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn();

// Checks that the current device is an sm_100 part and that the kernel's
// dynamic shared memory attribute has been raised on it (once per device).
int prepare_device(const void* kernel_fn, int smem_bytes, int* device_out);

// One kernel's per-device set-up state.  prepare_kernel() runs the set-up
// (sm_100 check, dynamic shared-memory limit) under a library mutex the first
// time the kernel is used on a device and publishes it through an atomic
// flag, so later calls -- from any thread -- only read the flag.
struct KernelPrep {
  std::atomic<bool> done[64] = {};
};
int prepare_kernel(KernelPrep& prep, const void* kernel_fn, int smem_bytes, int* device_out);

// Number of SMs of device dev (cached; 0 if the query failed).
int sm_count(int dev);

// Device-global status word written by kernels (fa::kDevTimeout ...).
int* device_status_ptr();

// Tensor map of 16-bit elements (bf16, or fp16 when f16) over a row-major
// [rows, cols] matrix (cols contiguous, row stride in elements), box =
// box_rows x 64 columns, 128B swizzle.
int make_tmap_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                 uint64_t row_stride_elems, uint32_t box_rows, uint32_t box_cols,
                 bool f16 = false);

// Tensor map of 16-bit elements over a [B, H, S, D] tensor with element
// strides (sb, sh, ss, 1): dims listed innermost first (D, S, H, B), box
// 64 x box_rows.  D may be below 64 (or between 64 and 128 for two boxes side
// by side): box columns past D read as zeros.
int make_tmap_bhsd(CUtensorMap* map, const void* base, int B, int H, int S, int D,
                   int64_t sb, int64_t sh, int64_t ss, uint32_t box_rows, bool f16 = false);

}  // namespace fa

// Shared host-side plumbing of libfa_b200: status strings, the driver entry
// point for tensor-map encoding, per-device preparation and the device-side
// status word.
#include <mutex>

#include "fa_internal.h"
#include "sm100_ptx.cuh"

namespace fa {

__device__ int g_fa_status = 0;

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
int* g_status_ptr[kMaxDevices] = {};
bool g_device_ok[kMaxDevices] = {};
bool g_device_checked[kMaxDevices] = {};
}  // namespace

EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

int prepare_device(const void* kernel_fn, int smem_bytes, int* device_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return FA_ERR_DEVICE;
  *device_out = dev;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_device_checked[dev]) {
      int major = 0, minor = 0;
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
      g_device_ok[dev] = (major == 10 && minor == 0);
      g_device_checked[dev] = true;
    }
  }
  if (!g_device_ok[dev]) return FA_ERR_DEVICE;
  // cudaFuncSetAttribute is per device and cheap to repeat; callers cache it.
  if (kernel_fn != nullptr &&
      cudaFuncSetAttribute(kernel_fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) !=
          cudaSuccess)
    return FA_ERR_CUDA;
  return FA_OK;
}

int prepare_kernel(KernelPrep& prep, const void* kernel_fn, int smem_bytes, int* device_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return FA_ERR_DEVICE;
  *device_out = dev;
  if (prep.done[dev].load(std::memory_order_acquire)) return FA_OK;
  static std::mutex prep_mu;
  std::lock_guard<std::mutex> lk(prep_mu);
  if (prep.done[dev].load(std::memory_order_relaxed)) return FA_OK;
  const int rc = prepare_device(kernel_fn, smem_bytes, &dev);
  if (rc != FA_OK) return rc;
  prep.done[dev].store(true, std::memory_order_release);
  return FA_OK;
}

int sm_count(int dev) {
  static std::atomic<int> n_sms[kMaxDevices] = {};
  if (dev < 0 || dev >= kMaxDevices) return 0;
  int n = n_sms[dev].load(std::memory_order_relaxed);
  if (n > 0) return n;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
    (void)cudaGetLastError();
    return 0;
  }
  n_sms[dev].store(n, std::memory_order_relaxed);
  return n;
}

int* device_status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_status_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_fa_status) != cudaSuccess) return nullptr;
    g_status_ptr[dev] = static_cast<int*>(p);
  }
  return g_status_ptr[dev];
}

int make_tmap_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                 uint64_t row_stride_elems, uint32_t box_rows, uint32_t box_cols, bool f16) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (enc == nullptr) return FA_ERR_DRIVER;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                   2, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FA_OK : FA_ERR_TMA;
}

int make_tmap_bhsd(CUtensorMap* map, const void* base, int B, int H, int S, int D, int64_t sb,
                   int64_t sh, int64_t ss, uint32_t box_rows, bool f16) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (enc == nullptr) return FA_ERR_DRIVER;
  // A size-1 dimension's stride is never used to address memory; give it a
  // legal value so the encoder's range checks pass for any caller stride.
  if (H == 1) sh = ss * S;
  if (B == 1) sb = sh * H;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)ss * 2, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
  cuuint32_t box[4] = {64, box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                   4, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FA_OK : FA_ERR_TMA;
}

}  // namespace fa

namespace fa {
namespace {

// One CTA waits on an mbarrier that nothing ever arrives on.  The bounded wait
// gives up after limit_ns, raises the CTA abort flag and records kDevTimeout
// in the device status word; the kernel then returns normally.
__global__ void wait_timeout_probe(int* status, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  mbar_wait_limit(smem_u32(&bar), 0, &abort_flag, status, limit_ns);
}

}  // namespace
}  // namespace fa

extern "C" int fa_selftest_wait_timeout(int limit_us, void* stream) {
  if (limit_us <= 0 || limit_us > 1000000) return FA_ERR_ARG;
  int dev = 0;
  int rc = fa::prepare_device(nullptr, 0, &dev);
  if (rc != FA_OK) return rc;
  int* status = fa::device_status_ptr();
  if (status == nullptr) return FA_ERR_CUDA;
  fa::wait_timeout_probe<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      status, static_cast<unsigned long long>(limit_us) * 1000ull);
  return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

extern "C" const char* fa_strerror(int status) {
  switch (status) {
    case FA_OK: return "success";
    case FA_ERR_NULL: return "a required pointer is NULL";
    case FA_ERR_SHAPE: return "invalid shape: every dimension must be positive and in range";
    case FA_ERR_HEAD_DIM:
      return "unsupported head dimension (attention supports D = 8 .. 128 in steps of 8)";
    case FA_ERR_ALIGN: return "pointer or stride is not 16-byte aligned (TMA requirement)";
    case FA_ERR_STRIDE: return "innermost stride must be 1 (contiguous last dimension)";
    case FA_ERR_TMA: return "cuTensorMapEncodeTiled rejected the tensor layout";
    case FA_ERR_LAUNCH: return "kernel launch failed";
    case FA_ERR_DRIVER: return "CUDA driver entry point cuTensorMapEncodeTiled unavailable";
    case FA_ERR_DEVICE: return "current device is not an sm_100 (B200-class) GPU";
    case FA_ERR_ARG: return "argument out of range";
    case FA_ERR_TIMEOUT: return "a kernel wait exceeded its time limit (device status)";
    case FA_ERR_CUDA: return "a CUDA runtime call failed";
    case FA_ERR_SCRATCH:
      return "M * N exceeds the fixed hidden buffer of fa_mlp_fwd_noalloc (8,388,608 elements)";
    default: return "unknown fa_status";
  }
}

extern "C" int fa_version(void) { return 100; }

extern "C" int fa_device_status(void) {
  int* p = fa::device_status_ptr();
  if (p == nullptr) return FA_ERR_CUDA;
  if (cudaDeviceSynchronize() != cudaSuccess) return FA_ERR_CUDA;
  int v = 0;
  if (cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return FA_ERR_CUDA;
  const int zero = 0;
  if (cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess)
    return FA_ERR_CUDA;
  return v == fa::kDevTimeout ? FA_ERR_TIMEOUT : FA_OK;
}

// Host-side runtime of the library: error strings, device checks and the
// per-device status word that kernels use to report bounded-wait timeouts and
// bad indices without trapping.
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include <cudaTypedefs.h>

#include "bs_common.cuh"
#include "bs_ptx.cuh"

namespace bs {
namespace {

thread_local char g_error[1024] = "";

// One status word per device (slot 0 is read by bs_device_status).  Kernels
// record the first error code with atomicCAS; the host reads and clears it.
__device__ int g_status_words[64];

constexpr int kMaxDevices = 64;
int* g_status_ptr[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};
int g_cc_major[kMaxDevices] = {};
std::mutex g_mu;

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

}  // namespace

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
}

const char* last_error() { return g_error; }

int* device_status_ptr() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_status_ptr[dev]) {
    void* p = nullptr;
    // The symbol name is only a host-side handle: the device address has to be
    // looked up once per device with that device current.
    if (cudaGetSymbolAddress(&p, g_status_words) != cudaSuccess) return nullptr;
    g_status_ptr[dev] = static_cast<int*>(p);
  }
  return g_status_ptr[dev];
}

int sm_count() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 148;
  if (!g_sm_count[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_sm_count[dev] = n > 0 ? n : 148;
  }
  return g_sm_count[dev];
}

int check_device() {
  const int dev = current_device();
  if (dev < 0) {
    set_error("no CUDA device is available");
    return BS_ERR_UNSUPPORTED;
  }
  if (dev < kMaxDevices && g_cc_major[dev] == 10) return BS_OK;
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0) {
    set_error("device %d is sm_%d%d; this library is built for sm_100a only", dev, major, minor);
    return BS_ERR_UNSUPPORTED;
  }
  if (dev < kMaxDevices) g_cc_major[dev] = major;
  return BS_OK;
}

namespace {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

}  // namespace

int make_map_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner,
                uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                CUtensorMapSwizzle sw) {
  auto fn = encode_fn();
  BS_REQUIRE(fn, BS_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  BS_REQUIRE(r == CUDA_SUCCESS, BS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return BS_OK;
}

int make_map_3d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, const uint64_t dims[3],
                const uint64_t strides[2], const uint32_t box[3], CUtensorMapSwizzle sw) {
  auto fn = encode_fn();
  BS_REQUIRE(fn, BS_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  cuuint64_t st[2] = {strides[0], strides[1]};
  cuuint32_t bx[3] = {box[0], box[1], box[2]};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, dt, 3, const_cast<void*>(base), d, st, bx, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  BS_REQUIRE(r == CUDA_SUCCESS, BS_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
  return BS_OK;
}

}  // namespace bs

extern "C" int bs_version(void) { return 1; }

extern "C" const char* bs_last_error_string(void) { return bs::last_error(); }

extern "C" int bs_device_status(int* out_status, int clear, void* stream) {
  using namespace bs;
  BS_ARG(out_status, "bs_device_status: null out_status");
  BS_TRY(check_device());
  int* p = device_status_ptr();
  BS_REQUIRE(p, BS_ERR_CUDA, "bs_device_status: cannot resolve the status word");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int v = 0;
  BS_CUDA(cudaMemcpyAsync(&v, p, sizeof(int), cudaMemcpyDeviceToHost, st));
  if (clear) BS_CUDA(cudaMemsetAsync(p, 0, sizeof(int), st));
  BS_CUDA(cudaStreamSynchronize(st));
  *out_status = v;
  return BS_OK;
}

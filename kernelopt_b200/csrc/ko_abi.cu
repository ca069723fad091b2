// Status reporting, device checks and tensor-map encoding shared by all entry points of libkernelopt.
#include <cstdio>
#include <mutex>
#include <string>

#include "ko_common.cuh"

namespace ko {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return static_cast<int>(e);
  }
  return KO_OK;
}

// One slot per device in a fixed array: callers keep the returned reference after the lock is released, while
// threads driving other devices may fill their own slots, so the storage must never move. A slot is written once,
// under the lock, after all four attributes were read; until then it reads as zeros.
const DeviceInfo& device_info() {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static DeviceInfo cache[kMaxDevices];
  static const DeviceInfo none;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return none;
  std::lock_guard<std::mutex> lock(mu);
  DeviceInfo& d = cache[dev];
  if (d.sm_count == 0) {
    DeviceInfo q;
    if (cudaDeviceGetAttribute(&q.sm_count, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&q.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&q.major, cudaDevAttrComputeCapabilityMajor, dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&q.minor, cudaDevAttrComputeCapabilityMinor, dev) == cudaSuccess && q.sm_count > 0)
      d = q;
  }
  return d;
}

int device_or_fail(const DeviceInfo** info, const char* who) {
  const DeviceInfo& d = device_info();
  if (d.sm_count <= 0)
    return fail(KO_ERR_UNSUPPORTED, std::string(who) + ": no usable CUDA device is current (attribute query failed)");
  *info = &d;
  return KO_OK;
}

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_2d_f32(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch_elems,
                     uint32_t box_rows, uint32_t box_cols, CUtensorMapSwizzle swizzle, const char* what) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(KO_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled is not available from the driver");
  if (!aligned16(base) || (pitch_elems * 4) % 16 != 0)
    return fail(KO_ERR_INVALID_ARGUMENT, std::string(what) + ": base must be 16-byte aligned and the row pitch a "
                                                             "multiple of 16 bytes");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch_elems * 4};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[160];
    snprintf(buf, sizeof buf, "%s: cuTensorMapEncodeTiled failed (CUresult %d)", what, static_cast<int>(r));
    return fail(KO_ERR_INVALID_ARGUMENT, buf);
  }
  return KO_OK;
}

int make_tmap_3d_f32(CUtensorMap* map, const void* base, uint64_t planes, uint64_t rows, uint64_t cols,
                     uint64_t row_pitch_elems, uint64_t plane_pitch_elems, uint32_t box_rows, uint32_t box_cols,
                     CUtensorMapSwizzle swizzle, const char* what) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(KO_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled is not available from the driver");
  if (!aligned16(base) || (row_pitch_elems * 4) % 16 != 0 || (plane_pitch_elems * 4) % 16 != 0 ||
      plane_pitch_elems == 0)
    return fail(KO_ERR_INVALID_ARGUMENT, std::string(what) + ": base must be 16-byte aligned and the pitches "
                                                             "non-zero multiples of 16 bytes");
  cuuint64_t dims[3] = {cols, rows, planes};
  cuuint64_t strides[2] = {row_pitch_elems * 4, plane_pitch_elems * 4};
  cuuint32_t box[3] = {box_cols, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[160];
    snprintf(buf, sizeof buf, "%s: cuTensorMapEncodeTiled failed (CUresult %d)", what, static_cast<int>(r));
    return fail(KO_ERR_INVALID_ARGUMENT, buf);
  }
  return KO_OK;
}

}  // namespace ko

extern "C" {

const char* ko_last_error_string(void) { return ko::g_last_error.c_str(); }

int ko_abi_version(void) { return 2; }

int ko_check_device(void) {
  const ko::DeviceInfo& d = ko::device_info();
  if (d.major != 10)
    return ko::fail(KO_ERR_UNSUPPORTED, "libkernelopt is built for sm_100a (B200); current device is sm_" +
                                            std::to_string(d.major) + std::to_string(d.minor));
  return KO_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------------------
// ko_wait_probe: the bounded on-chip wait of the tcgen05 kernels, run on an mbarrier that nothing arrives on.
// Warp 0 waits (mbar_wait_for, the code path behind every mbar_wait) until limit_ns pass and raises the CTA's
// abort flag; warp 1 waits on the same barrier with the full limit and must leave as soon as it sees the flag;
// thread 0 then writes KO_ERR_DEVICE_TIMEOUT to *dev_status, as the kernels do. Nothing faults and the
// context stays usable: this is how the timeout path is exercised in tests.
// ---------------------------------------------------------------------------------------------------------
namespace {
__global__ void wait_probe_kernel(uint64_t limit_ns, int* dev_status) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    kodev::mbar_init(&bar, 1);
    abort_flag = 0;
    kodev::fence_barrier_init();
  }
  __syncthreads();
  volatile int* abort = &abort_flag;
  bool ok = true;
  if (threadIdx.x < 32) ok = kodev::mbar_wait_for(&bar, 0, abort, limit_ns);
  else ok = kodev::mbar_wait(&bar, 0, abort);
  __syncthreads();
  if (threadIdx.x == 0 && (!ok || *abort) && dev_status) atomicExch(dev_status, KO_ERR_DEVICE_TIMEOUT);
}
}  // namespace

extern "C" int ko_wait_probe(int64_t limit_ns, int* dev_status, ko_stream_t stream) {
  if (limit_ns < 0 || limit_ns > 10000000000ll || !dev_status)
    return ko::fail(KO_ERR_INVALID_ARGUMENT, "ko_wait_probe: need 0 <= limit_ns <= 10 s and a status word");
  wait_probe_kernel<<<1, 64, 0, reinterpret_cast<cudaStream_t>(stream)>>>(static_cast<uint64_t>(limit_ns), dev_status);
  return ko::check_launch("ko_wait_probe");
}

// Host runtime of the library: thread-local error messages, the per-device status word,
// cached device attributes and TMA tensor-map encoding.
#include <cudaTypedefs.h>

#include <mutex>
#include <string>

#include "common.cuh"

namespace sa {

namespace {
thread_local std::string t_last_error;
constexpr int kMaxDevices = 64;
}  // namespace

void set_error(const std::string& msg) { t_last_error = msg; }

int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SA_ELAUNCH, std::string(what) + ": " + cudaGetErrorString(e));
  return SA_OK;
}

// One status word per device (module-scope __device__ memory, zero at load).
__device__ unsigned g_device_status_word;

unsigned* device_status_ptr() {
  static unsigned* ptrs[kMaxDevices] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    set_error("device status word: no current device");
    return nullptr;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("device status word: device index " + std::to_string(dev) + " out of range");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_device_status_word);
    if (e != cudaSuccess) {
      // keep the message, and clear the runtime's sticky last error so that a later
      // check_launch does not report it against an unrelated kernel
      cudaGetLastError();
      set_error(std::string("device status word address: ") + cudaGetErrorString(e));
      return nullptr;
    }
    ptrs[dev] = static_cast<unsigned*>(p);
  }
  return ptrs[dev];
}

int check_stream_device(void* stream, const char* what) {
  if (!stream) return SA_OK;  // the legacy default stream belongs to the current device
  // a stream being captured into a graph is not queried (the capture holds the device)
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(static_cast<cudaStream_t>(stream), &cs) != cudaSuccess) {
    cudaGetLastError();
    return fail(SA_EINVAL, std::string(what) + ": not a valid CUDA stream");
  }
  if (cs != cudaStreamCaptureStatusNone) return SA_OK;
  int dev = 0, sdev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return fail(SA_ELAUNCH, std::string(what) + ": no current device");
  }
  if (cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &sdev) != cudaSuccess) {
    cudaGetLastError();
    return fail(SA_EINVAL, std::string(what) + ": not a valid CUDA stream");
  }
  if (sdev != dev)
    return fail(SA_EINVAL, std::string(what) + ": the stream belongs to device " +
                               std::to_string(sdev) + " but the current device is " +
                               std::to_string(dev) + "; make the stream's device current");
  return SA_OK;
}

// A second stream (and a fork / join event pair) per host thread and device, created on
// first use, for independent launches inside one entry point (the backward's preparation
// phase).  It has the highest stream priority: its small latency-bound kernels get SM slots
// ahead of a wide kernel running beside them on the caller's stream.  This is the library's
// only host-side resource besides the read-only attribute caches; every entry point joins
// the side stream back into the caller's stream before it returns, and
// sa_release_thread_resources() destroys the calling thread's streams and events.
namespace {
struct Side {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
thread_local Side t_side[kMaxDevices];
}  // namespace

int side_stream(cudaStream_t* out, cudaEvent_t* fork, cudaEvent_t* join) {
  Side* side = t_side;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(SA_ELAUNCH, "side stream: no current device");
  Side& d = side[dev];
  if (!d.s) {
    int least = 0, greatest = 0;
    cudaDeviceGetStreamPriorityRange(&least, &greatest);
    if (cudaStreamCreateWithPriority(&d.s, cudaStreamNonBlocking, greatest) != cudaSuccess ||
        cudaEventCreateWithFlags(&d.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&d.join, cudaEventDisableTiming) != cudaSuccess)
      return check_launch("side stream creation");
  }
  *out = d.s;
  *fork = d.fork;
  *join = d.join;
  return SA_OK;
}

int device_sm_count() {
  static int counts[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  if (!counts[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    counts[dev] = n > 0 ? n : 148;
  }
  return counts[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int make_tmap_4d(CUtensorMap* map, const void* base, int dtype, int64_t Z, int64_t Hh, int64_t N,
                 int64_t D, const int64_t* strides, uint32_t box_d, uint32_t box_n) {
  auto fn = encode_fn();
  if (!fn) return fail(SA_ELAUNCH, "cuTensorMapEncodeTiled is unavailable");
  const int64_t esz = dtype == SA_F32 ? 4 : 2;
  if (strides[3] != 1) return fail(SA_EUNSUPPORTED, "innermost (head_dim) stride must be 1");
  if (reinterpret_cast<uintptr_t>(base) % 16)
    return fail(SA_EUNSUPPORTED, "tensor base address must be 16-byte aligned");
  for (int i = 0; i < 3; ++i)
    if ((strides[i] * esz) % 16)
      return fail(SA_EUNSUPPORTED, "tensor strides must be multiples of 16 bytes");
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)N, (cuuint64_t)Hh, (cuuint64_t)Z};
  cuuint64_t gstr[3] = {(cuuint64_t)(strides[2] * esz), (cuuint64_t)(strides[1] * esz),
                        (cuuint64_t)(strides[0] * esz)};
  // Size-1 dims may carry any stride; TMA still wants a valid (non-zero, aligned) one.
  if (N == 1) gstr[0] = (cuuint64_t)(D * esz);
  if (Hh == 1) gstr[1] = gstr[0] * (cuuint64_t)N;
  if (Z == 1) gstr[2] = gstr[1] * (cuuint64_t)Hh;
  cuuint32_t box[4] = {box_d, box_n, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUtensorMapDataType dt = dtype == SA_BF16  ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                           : dtype == SA_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                             : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUresult r = fn(map, dt, 4, const_cast<void*>(base), dims, gstr, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SA_EUNSUPPORTED, "cuTensorMapEncodeTiled failed (code " +
                                                           std::to_string((int)r) + ")");
  return SA_OK;
}

}  // namespace sa

extern "C" {

const char* sa_last_error(void) { return sa::t_last_error.c_str(); }

int sa_abi_version(void) { return 3; }

// Destroy the side streams and events the calling thread created (one set per device it
// used); the next backward call on this thread creates them again.  Synchronises each of
// those streams first, so it must not be called while a capture uses them.
int sa_release_thread_resources(void) {
  int prev = 0;
  const bool had_dev = cudaGetDevice(&prev) == cudaSuccess;
  int rc = SA_OK;
  for (int d = 0; d < sa::kMaxDevices; ++d) {
    sa::Side& s = sa::t_side[d];
    if (!s.s) continue;
    if (cudaSetDevice(d) != cudaSuccess || cudaStreamSynchronize(s.s) != cudaSuccess ||
        cudaStreamDestroy(s.s) != cudaSuccess || cudaEventDestroy(s.fork) != cudaSuccess ||
        cudaEventDestroy(s.join) != cudaSuccess)
      rc = sa::check_launch("release side stream");
    s = sa::Side{};
  }
  if (had_dev) cudaSetDevice(prev);
  return rc;
}

// Read (and optionally clear) the current device's status word.  Synchronises the device.
int sa_read_device_status(int reset, unsigned* value) {
  unsigned* p = sa::device_status_ptr();
  if (!p || !value) return sa::fail(SA_ELAUNCH, "device status word unavailable");
  if (cudaMemcpy(value, p, sizeof(unsigned), cudaMemcpyDeviceToHost) != cudaSuccess)
    return sa::check_launch("read device status");
  if (reset && cudaMemset(p, 0, sizeof(unsigned)) != cudaSuccess)
    return sa::check_launch("reset device status");
  return SA_OK;
}

}  // extern "C"

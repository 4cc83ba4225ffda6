// Host-side plumbing shared by every entry point of libbw_ops.so: status
// codes and per-thread error detail, device checks, TMA tensor-map encoding
// (driver entry point fetched through the runtime, so the library does not
// link libcuda directly) and the device-side status word written by kernels
// whose bounded waits expire.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "common.cuh"

namespace bw {

__device__ int g_status = 0;
__device__ TraceState g_trace = {nullptr, 0u, 0u};
__device__ long long g_wait_limit_cycles = static_cast<long long>(BW_WAIT_LIMIT_NS) * 5 / 2;

static thread_local char t_msg[512] = {0};

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
  va_end(ap);
  return status;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return BW_OK;
  return fail(BW_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int check_launch(const char* what) { return check_cuda(cudaGetLastError(), what); }

struct DevInfo {
  int sms = 0;
  int major = 0;
  int minor = 0;
};

static DevInfo dev_info(int dev) {
  static DevInfo cache[64];
  static std::once_flag once[64];
  std::call_once(once[dev & 63], [dev] {
    DevInfo d;
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev);
    cache[dev & 63] = d;
  });
  return cache[dev & 63];
}

int num_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  const int s = dev_info(dev).sms;
  return s > 0 ? s : 148;
}

int require_sm100() {
  int dev = 0;
  if (cudaError_t e = cudaGetDevice(&dev)) return check_cuda(e, "cudaGetDevice");
  const DevInfo d = dev_info(dev);
  if (d.major != 10 || d.minor != 0)
    return fail(BW_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a (B200) only", dev,
                d.major, d.minor);
  return BW_OK;
}

int dtype_size(int dtype) { return dtype == BW_DTYPE_F32 ? 4 : 2; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
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

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t rows, uint64_t cols,
                 uint64_t ld_bytes, uint32_t box_rows, uint32_t box_cols, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(BW_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled is unavailable from the driver");
  const cuuint64_t gdim[2] = {cols, rows};
  const cuuint64_t gstride[1] = {ld_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = fn(map, dt, 2, const_cast<void*>(base), gdim, gstride, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(BW_ERR_INVALID_ARGUMENT,
                "cuTensorMapEncodeTiled failed (%d): rows=%llu cols=%llu ld=%llu box=%ux%u base=%p", (int)r,
                (unsigned long long)rows, (unsigned long long)cols, (unsigned long long)ld_bytes, box_rows,
                box_cols, base);
  return BW_OK;
}

}  // namespace bw

extern "C" const char* bw_status_string(int status) {
  switch (status) {
    case BW_OK: return "ok";
    case BW_ERR_INVALID_ARGUMENT: return "invalid argument";
    case BW_ERR_WORKSPACE: return "workspace missing or too small";
    case BW_ERR_CUDA: return "CUDA runtime error";
    case BW_ERR_DEVICE_TIMEOUT: return "device wait timed out";
    case BW_ERR_UNSUPPORTED: return "unsupported device or feature";
    default: return "unknown status";
  }
}

extern "C" const char* bw_last_error(void) { return bw::t_msg; }

extern "C" int bw_version(void) { return 1 * 10000 + 0 * 100 + 0; }

extern "C" int bw_set_wait_limit_ns(uint64_t ns) {
  using namespace bw;
  if (ns == 0 || ns > (1ull << 60) / 5)
    return fail(BW_ERR_INVALID_ARGUMENT, "wait limit must be in (0, 2^60/5) ns (got %llu)", (unsigned long long)ns);
  const long long cycles = static_cast<long long>(ns * 5 / 2);
  return check_cuda(cudaMemcpyToSymbol(g_wait_limit_cycles, &cycles, sizeof(cycles)), "set wait limit");
}

extern "C" int bw_get_wait_limit_ns(uint64_t* ns) {
  using namespace bw;
  if (!ns) return fail(BW_ERR_INVALID_ARGUMENT, "null pointer");
  long long cycles = 0;
  if (int s = check_cuda(cudaMemcpyFromSymbol(&cycles, g_wait_limit_cycles, sizeof(cycles)), "read wait limit"))
    return s;
  *ns = static_cast<uint64_t>(cycles) * 2 / 5;
  return BW_OK;
}

extern "C" int bw_trace_enable(void* buffer, size_t bytes) {
  using namespace bw;
  TraceState t = {nullptr, 0u, 0u};
  if (buffer != nullptr) {
    if (bytes < 128)
      return fail(BW_ERR_INVALID_ARGUMENT, "trace buffer of %zu bytes holds no record (128 bytes)", bytes);
    if (reinterpret_cast<uintptr_t>(buffer) % 8 != 0)
      return fail(BW_ERR_INVALID_ARGUMENT, "trace buffer must be 8-byte aligned");
    t.buf = static_cast<unsigned long long*>(buffer);
    t.records = static_cast<unsigned int>(bytes / 128 > 0x7FFFFFFFu ? 0x7FFFFFFFu : bytes / 128);
  }
  return check_cuda(cudaMemcpyToSymbol(g_trace, &t, sizeof(t)), "set trace buffer");
}

extern "C" int bw_trace_records(unsigned int* records) {
  using namespace bw;
  if (!records) return fail(BW_ERR_INVALID_ARGUMENT, "null pointer");
  TraceState t;
  if (int s = check_cuda(cudaMemcpyFromSymbol(&t, g_trace, sizeof(t)), "read trace state")) return s;
  *records = t.next < t.records ? t.next : t.records;
  return BW_OK;
}

extern "C" int bw_device_status(int clear, int* detail, void* stream) {
  using namespace bw;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int s = check_cuda(cudaStreamSynchronize(st), "cudaStreamSynchronize")) return s;
  int v = 0;
  if (int s = check_cuda(cudaMemcpyFromSymbol(&v, g_status, sizeof(int)), "read device status")) return s;
  if (detail) *detail = v;
  if (clear && v != 0) {
    const int zero = 0;
    if (int s = check_cuda(cudaMemcpyToSymbol(g_status, &zero, sizeof(int)), "clear device status")) return s;
  }
  if (v != 0) return fail(BW_ERR_DEVICE_TIMEOUT, "a kernel's bounded wait expired at site %d", v);
  return BW_OK;
}

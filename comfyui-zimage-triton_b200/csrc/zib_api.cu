// Library-level entry points: version, status strings, error reporting,
// device checks.
#include "zib_common.cuh"

#include <stdarg.h>
#include <stdio.h>

static thread_local char g_last_error[512] = "";

void zib_set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int zib_check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    zib_set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
    return ZIB_ERR_LAUNCH;
  }
  return ZIB_OK;
}

extern "C" int zib_version(void) { return 100; }  // 0.1.0

extern "C" const char* zib_status_string(int status) {
  switch (status) {
    case ZIB_OK: return "ok";
    case ZIB_ERR_INVALID_ARG: return "invalid argument";
    case ZIB_ERR_ALIGNMENT: return "misaligned operand";
    case ZIB_ERR_UNSUPPORTED: return "unsupported device or feature";
    case ZIB_ERR_LAUNCH: return "CUDA launch error";
    case ZIB_ERR_TOO_LARGE: return "size exceeds the supported maximum";
    case ZIB_ERR_TIMEOUT: return "bounded device wait expired";
    default: return "unknown status";
  }
}

extern "C" const char* zib_last_error(void) { return g_last_error; }

// per-translation-unit device error words (see zib_async.cuh)
int zib_err_read_clear_gemm();
void zib_gemm_split_reset();
int zib_err_read_clear_rows();

extern "C" int zib_device_error_read_clear(void) {
  // every stream of the device, non-blocking ones included, has finished before the
  // word is read (and before any counter is re-zeroed below)
  cudaDeviceSynchronize();
  cudaGetLastError();
  int a = zib_err_read_clear_gemm();
  int b = zib_err_read_clear_rows();
  if (a) zib_gemm_split_reset();  // a stopped GEMM may have left split-K counters mid-count
  return a ? a : b;
}

extern "C" int zib_device_check(int dev) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    zib_set_error("no CUDA device visible");
    return ZIB_ERR_UNSUPPORTED;
  }
  if (dev < 0 || dev >= n) {
    zib_set_error("device %d out of range (%d devices)", dev, n);
    return ZIB_ERR_INVALID_ARG;
  }
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0) {
    zib_set_error("device %d is sm_%d%d; this library is built for sm_100a (B200) only", dev, major, minor);
    return ZIB_ERR_UNSUPPORTED;
  }
  return ZIB_OK;
}

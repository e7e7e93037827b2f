// Error reporting and device status for the kvquant_b200 C ABI (part of the kvq_lib.cu unity build).
#pragma once
#include "kvq_common.cuh"

namespace kvq {

static thread_local char t_error[512] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_error, sizeof(t_error), fmt, ap);
  va_end(ap);
}

void clear_error() { t_error[0] = 0; }


int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: CUDA error %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
    return KVQ_ERR_CUDA;
  }
  return KVQ_OK;
}

}  // namespace kvq

extern "C" const char* kvq_last_error(void) { return kvq::t_error; }

extern "C" int kvq_version(void) { return 100; }

extern "C" int kvq_check_status(void* stream) {
  cudaStream_t s = kvq::as_stream(stream);
  int host = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&host, kvq::g_status, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    kvq::set_error("kvq_check_status: %s", cudaGetErrorString(e));
    return KVQ_ERR_CUDA;
  }
  if (host != 0) {
    const int zero = 0;
    cudaMemcpyToSymbolAsync(kvq::g_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
    cudaStreamSynchronize(s);
    kvq::set_error("kernel reported invalid input (status 0x%x): index out of range", host);
    return KVQ_ERR_INVALID;
  }
  return KVQ_OK;
}

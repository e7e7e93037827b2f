// kvq_value_output_noalloc: the value kernel (p.V over the packed value cache)
// with its scratch taken from a fixed array owned by the library instead of a
// caller workspace.
//
// Who needs it: a caller that has no device allocator of its own to hand the
// library a workspace -- e.g. a host runtime binding the C ABI through a plain
// FFI, or a decode loop that must not call cudaMalloc between steps (it
// synchronizes the device) and keeps no buffer of its own for this call.
//
// Scratch: kNoAllocScratchBytes (4 MiB) in a file-scope __device__ array, one
// copy per device (each device's module has its own). The call needs
// kvq_value_output_workspace(B, n_heads, group, T) bytes of it -- the split-K
// partial sums (n_splits x B*n_heads*group x 129 floats) and one float per
// batch row -- and returns KVQ_ERR_INVALID with a message when that is more.
// Nothing in the scratch has to start at zero: every byte the call reads was
// written earlier in the same call.
//
// Set-up: the first call on a device looks the array's address up with
// cudaGetSymbolAddress (with that device current) and caches it; make that
// first call before any stream capture begins. The cached address belongs to
// the device's primary context: it does not survive cudaDeviceReset (which
// unloads the module and its array), and a caller that runs the library
// under a context of its own other than the primary one must not use this
// entry point.
//
// Concurrency: all calls on one device share the one array. Two calls whose
// work overlaps in time (different streams, or different host threads with
// no ordering between their streams) race on it and may produce wrong
// outputs; calls issued in order on one stream are safe.
#pragma once
#include <mutex>

#include "kvq_decode.cuh"

namespace kvq {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[kNoAllocMaxDevices];  // per-device address, set on first use

// Device address of the current device's copy of the scratch array.
static int noalloc_scratch(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("value_output_noalloc: cudaGetDevice failed: %s", cudaGetErrorString(e));
    return KVQ_ERR_CUDA;
  }
  if (dev < 0 || dev >= kNoAllocMaxDevices) {
    set_error("value_output_noalloc: device %d is beyond the %d devices supported", dev,
              kNoAllocMaxDevices);
    return KVQ_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress((void**)&ptr, g_noalloc_scratch);  // device `dev` is current
    if (e != cudaSuccess || !ptr) {
      set_error("value_output_noalloc: cudaGetSymbolAddress on device %d failed: %s", dev,
                cudaGetErrorString(e));
      return KVQ_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return KVQ_OK;
}

}  // namespace kvq

extern "C" int kvq_value_output_noalloc(const uint8_t* codes, const uint32_t* out_ent,
                                        const int32_t* out_ptr, const float* v_scale,
                                        const float* v_zero, int64_t ld_stats,
                                        const void* v_sink, const float* codebook, int bits,
                                        const float* probs, int64_t B, int64_t n_heads,
                                        int64_t group, int64_t T, int64_t nt_cap, void* out,
                                        void* stream) {
  using namespace kvq;
  clear_error();
  int rc = check_decode_shape("value_output_noalloc", B, n_heads, group, T, nt_cap);
  if (rc) return rc;
  const size_t need = value_ws(B, n_heads, group, T);
  if (need > kNoAllocScratchBytes) {
    set_error("value_output_noalloc: this shape needs %zu bytes of scratch, more than the "
              "library's fixed %zu; use kvq_value_output with a caller workspace",
              need, kNoAllocScratchBytes);
    return KVQ_ERR_INVALID;
  }
  void* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return value_impl(codes, out_ent, out_ptr, v_scale, v_zero, ld_stats, v_sink, codebook, bits,
                    probs, B, n_heads, group, T, nt_cap, out, scratch, kNoAllocScratchBytes,
                    as_stream(stream));
}

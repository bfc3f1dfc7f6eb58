// Helpers shared by the translation units of libggo_b200.so (not part of the public ABI).
#pragma once

#include "ggo.h"

#include <atomic>
#include <cstdint>

#include <cuda_runtime_api.h>

namespace ggo {

// Last CUDA runtime error (or 100000 + driver CUresult) seen by a failing call on this thread,
// reported by ggo_last_cuda_error_string().
inline thread_local int g_last_cuda_error = 0;

inline int cuda_fail(int code) {
  g_last_cuda_error = code;
  return GGO_ERR_CUDA;
}

// Kernels launched by this library in this process (ggo_kernel_launches()).
inline std::atomic<uint64_t> g_kernel_launches{0};

// Called right after every kernel launch.
inline int check_launch() {
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? GGO_OK : cuda_fail(static_cast<int>(e));
}

// Maps a device-side error word (GgoWorkspace::error) to a public status code.
inline int device_error_to_status(int code) {
  if (code == 0) return GGO_OK;
  if (code >= 101 && code <= 109) return GGO_ERR_DEVICE_TIMEOUT;  // 104: expert-parallel peer wait
  if (code == 110) return GGO_ERR_COUNT_MISMATCH;
  if (code == 111) return GGO_ERR_NEGATIVE_COUNT;
  return GGO_ERR_CUDA;
}

}  // namespace ggo

// Helpers shared by the translation units of libggo_b200.so (not part of the public ABI).
#pragma once

#include "ggo.h"

namespace ggo {

// Maps a device-side error word (GgoWorkspace::error) to a public status code.
inline int device_error_to_status(int code) {
  if (code == 0) return GGO_OK;
  if (code >= 101 && code <= 109) return GGO_ERR_DEVICE_TIMEOUT;
  if (code == 110) return GGO_ERR_COUNT_MISMATCH;
  if (code == 111) return GGO_ERR_NEGATIVE_COUNT;
  return GGO_ERR_CUDA;
}

}  // namespace ggo

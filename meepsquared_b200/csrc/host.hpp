// Host-side helpers shared by the entry points of libmeep2b: device binding, launch checks, tensor maps.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/meep2b.h"

namespace meep2b {

// Makes the stream's device current for this thread's runtime (the library links its own CUDA runtime, whose
// current device is independent of the caller's). Returns MEEP2B_OK or MEEP2B_ERR_LAUNCH.
int bind_stream_device(cudaStream_t stream);

// MEEP2B_OK, or MEEP2B_ERR_LAUNCH (and the error cleared) when the last launch failed.
int launch_status();

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link-time dependency on libcuda).
// dims / strides in elements / bytes, innermost first; strides[0] is the stride of dimension 1.
int encode_tiled(CUtensorMap* map, CUtensorMapDataType type, uint32_t rank, const void* base, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

}  // namespace meep2b

#define MEEP2B_TRY(expr)             \
  do {                               \
    int _st = (expr);                \
    if (_st != MEEP2B_OK) return _st; \
  } while (0)

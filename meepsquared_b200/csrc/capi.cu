// Library-level entry points of libmeep2b: version, status strings, the device check and the device error word.
#include <cstdio>

#include "common.cuh"
#include "host.hpp"

namespace meep2b {

int bind_stream_device(cudaStream_t stream) {
  int want = -1;
  if (stream != nullptr) {
    // a stream being captured into a CUDA graph is not queried for its device (the query is not a capturable
    // operation); the caller captures on the current device
    cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &capturing) != cudaSuccess) {
      cudaGetLastError();
      return MEEP2B_ERR_LAUNCH;
    }
    if (capturing != cudaStreamCaptureStatusNone) return MEEP2B_OK;
    if (cudaStreamGetDevice(stream, &want) != cudaSuccess) {
      cudaGetLastError();
      return MEEP2B_ERR_LAUNCH;
    }
  } else if (cudaGetDevice(&want) != cudaSuccess) {
    cudaGetLastError();
    return MEEP2B_ERR_LAUNCH;
  }
  // cudaSetDevice also makes the device's primary context current on this thread. The tensor-map encoding is a
  // driver call and needs it: a thread that has made no runtime call yet (autograd runs the backward pass on its
  // own thread) has no current context, and the encoding would fail with an invalid-context error.
  if (cudaSetDevice(want) != cudaSuccess) {
    cudaGetLastError();
    return MEEP2B_ERR_LAUNCH;
  }
  return MEEP2B_OK;
}

int launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return MEEP2B_ERR_LAUNCH;
  }
  return MEEP2B_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    } else {
      cudaGetLastError();
    }
  }
  return fn;
}

int encode_tiled(CUtensorMap* map, CUtensorMapDataType type, uint32_t rank, const void* base, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return MEEP2B_ERR_LAUNCH;
  if (!aligned16(base)) return MEEP2B_ERR_ALIGN;
  for (uint32_t i = 0; i + 1 < rank; ++i)
    if (strides_bytes[i] % 16 != 0) return MEEP2B_ERR_ALIGN;
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, type, rank, const_cast<void*>(base), reinterpret_cast<const cuuint64_t*>(dims),
                  reinterpret_cast<const cuuint64_t*>(strides_bytes), reinterpret_cast<const cuuint32_t*>(box),
                  elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MEEP2B_OK : MEEP2B_ERR_ALIGN;
}

}  // namespace meep2b

extern "C" {

const char* meep2b_version(void) { return "meep2b 0.1.0 (sm_100a)"; }

const char* meep2b_status_string(int status) {
  switch (status) {
    case MEEP2B_OK: return "ok";
    case MEEP2B_ERR_SHAPE: return "sizes that do not fit together";
    case MEEP2B_ERR_DTYPE: return "an element type the entry point does not take";
    case MEEP2B_ERR_LAUNCH: return "a CUDA runtime or driver call failed";
    case MEEP2B_ERR_TIMEOUT: return "a bounded device-side wait ran out";
    case MEEP2B_ERR_UNSUPPORTED: return "a combination the kernels do not implement";
    case MEEP2B_ERR_ALIGN: return "a pointer or row stride TMA cannot address (16-byte rule)";
    case MEEP2B_ERR_DEVICE: return "not a compute capability 10.0 GPU";
    default: return "unknown status";
  }
}

int meep2b_device_ok(int device) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
    cudaGetLastError();
    return MEEP2B_ERR_DEVICE;
  }
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess) {
    cudaGetLastError();
    return MEEP2B_ERR_DEVICE;
  }
  return (major == 10 && minor == 0) ? MEEP2B_OK : MEEP2B_ERR_DEVICE;
}

int meep2b_device_error(int device, int* code) {
  if (cudaSetDevice(device) != cudaSuccess) {
    cudaGetLastError();
    return MEEP2B_ERR_LAUNCH;
  }
  int value = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&value, meep2b::g_device_error, sizeof(int)) != cudaSuccess ||
      cudaMemcpyToSymbol(meep2b::g_device_error, &zero, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return MEEP2B_ERR_LAUNCH;
  }
  if (code) *code = value;
  return MEEP2B_OK;
}

int meep2b_sm_count(int device, int* count) {
  if (cudaDeviceGetAttribute(count, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) {
    cudaGetLastError();
    return MEEP2B_ERR_LAUNCH;
  }
  return MEEP2B_OK;
}

}  // extern "C"

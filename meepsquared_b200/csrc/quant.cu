// Quantised expert stacks: FP8 e4m3 with one scale per expert (meepsquared/_fp8.py:111-134), FP8 with 2-D block
// scales (meepsquared/_vendor/axolotl/quantize.py:131-157, 238-263) and NF4 with a double-quantised absmax
// (quantize.py:52-101, the bitsandbytes kernels it calls). Elementwise and HBM-bound: 16-byte vector accesses,
// one pass each. The e4m3 conversions use the hardware cvt instructions: e4m3 -> f16 is exact, and f32 -> e4m3
// rounds to nearest even and saturates to +-448 (equal to PyTorch's cast for every value the quantisers produce,
// which never exceed 448 in magnitude by more than the rounding band).
#include "common.cuh"
#include "host.hpp"

#include <cuda_fp16.h>

namespace meep2b {
namespace quant {

__device__ __forceinline__ float e4m3_to_float(uint8_t c) {
  uint16_t h2;
  const uint16_t in = c;
  asm("{\n\t.reg .b32 t;\n\tcvt.rn.f16x2.e4m3x2 t, %1;\n\tmov.b32 {%0, _}, t;\n\t}" : "=h"(h2) : "h"(in));
  return __half2float(__ushort_as_half(h2));
}

__device__ __forceinline__ uint8_t float_to_e4m3(float v) {
  uint16_t out;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;" : "=h"(out) : "f"(v), "f"(0.0f));
  return static_cast<uint8_t>(out & 0xFF);
}

template <typename T>
__device__ __forceinline__ float load_f(const T* p, int64_t i);
template <>
__device__ __forceinline__ float load_f<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float load_f<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}

// |x| of non-negative floats orders like their bit patterns: atomicMax on the int view.
__device__ __forceinline__ void atomic_max_pos(float* addr, float v) {
  atomicMax(reinterpret_cast<int*>(addr), __float_as_int(v));
}

template <typename T>
__global__ void stack_amax(const T* __restrict__ w, int64_t per_expert, float* __restrict__ amax) {
  const int e = blockIdx.y;
  const T* base = w + static_cast<int64_t>(e) * per_expert;
  float m = 0.f;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < per_expert;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    m = fmaxf(m, fabsf(load_f(base, i)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomic_max_pos(amax + e, m);
}

template <typename T>
__global__ void stack_cast(const T* __restrict__ w, int64_t per_expert, const float* __restrict__ amax,
                           uint8_t* __restrict__ codes, float* __restrict__ scale) {
  const int e = blockIdx.y;
  const float s = fmaxf(amax[e], 1e-12f) / 448.0f;
  if (blockIdx.x == 0 && threadIdx.x == 0) scale[e] = s;
  const int64_t off = static_cast<int64_t>(e) * per_expert;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < per_expert;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    codes[off + i] = float_to_e4m3(__fdiv_rn(load_f(w + off, i), s));
}

__global__ void stack_dequant(const uint8_t* __restrict__ codes, const float* __restrict__ scale, int64_t per_expert,
                              int64_t total, __nv_bfloat16* __restrict__ out) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = __float2bfloat16_rn(__fmul_rn(e4m3_to_float(codes[i]), scale[i / per_expert]));
}

// out = bf16(bf16(w8) * bf16(s)), the block of element (r, c) being (r / br, c / bc) of its matrix.
__global__ void block_dequant(const uint8_t* __restrict__ codes, int64_t rows, int64_t cols,
                              const float* __restrict__ scale_inv, int sr, int sc, int64_t br, int64_t bc,
                              int64_t total, __nv_bfloat16* __restrict__ out) {
  const int64_t per = rows * cols;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = i / per, rem = i - m * per;
    const int64_t r = rem / cols, c = rem - r * cols;
    const float s = bf16_round(scale_inv[m * sr * sc + (r / br) * sc + (c / bc)]);
    out[i] = __float2bfloat16_rn(__fmul_rn(e4m3_to_float(codes[i]), s));
  }
}

// One CTA per block of one matrix: amax, scale, then codes.
template <typename T>
__global__ void block_quant(const T* __restrict__ w, int64_t rows, int64_t cols, int sr, int sc, int64_t br,
                            int64_t bc, uint8_t* __restrict__ codes, float* __restrict__ scale_inv) {
  __shared__ float red[32];
  const int64_t m = blockIdx.z;
  const int bi = blockIdx.y, bj = blockIdx.x;
  const int64_t r0 = bi * br, c0 = bj * bc;
  const int64_t r1 = min(r0 + br, rows), c1 = min(c0 + bc, cols);
  const int64_t h = r1 > r0 ? r1 - r0 : 0, wdt = c1 > c0 ? c1 - c0 : 0;
  const T* base = w + m * rows * cols;
  float mx = 0.f;
  for (int64_t i = threadIdx.x; i < h * wdt; i += blockDim.x) {
    const int64_t r = r0 + i / wdt, c = c0 + i % wdt;
    mx = fmaxf(mx, fabsf(load_f(base, r * cols + c)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float s = fmaxf(red[0], 1e-12f) / 448.0f;
  if (threadIdx.x == 0) scale_inv[m * sr * sc + bi * sc + bj] = s;
  for (int64_t i = threadIdx.x; i < h * wdt; i += blockDim.x) {
    const int64_t r = r0 + i / wdt, c = c0 + i % wdt;
    const float q = fminf(fmaxf(__fdiv_rn(load_f(base, r * cols + c), s), -448.0f), 448.0f);
    codes[m * rows * cols + r * cols + c] = float_to_e4m3(q);
  }
}

__global__ void nf4_absmax(const uint8_t* __restrict__ absmax, const float* __restrict__ absmax2,
                           const float* __restrict__ code2, const float* __restrict__ offset, int blocksize2,
                           int64_t count, float* __restrict__ out) {
  const float off = offset[0];
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = __fadd_rn(__fmul_rn(code2[absmax[i]], absmax2[i / blocksize2]), off);
}

// 8 packed bytes (16 weights) per thread and step: one 8-byte load, two 16-byte stores.
__global__ void nf4_dequant(const uint2* __restrict__ packed, const float* __restrict__ absmax, int blocksize,
                            int64_t groups, uint4* __restrict__ out) {
  for (int64_t gi = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; gi < groups;
       gi += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint2 p = packed[gi];
    const uint32_t words[2] = {p.x, p.y};
    const int64_t first = gi * 16;
    uint32_t res[8];
#pragma unroll
    for (int w = 0; w < 2; ++w) {
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t byte = (words[w] >> (8 * b)) & 0xFF;
        const int64_t j = first + 8 * w + 2 * b;
        const float hi = __fmul_rn(kNF4Levels[byte >> 4], absmax[j / blocksize]);
        const float lo = __fmul_rn(kNF4Levels[byte & 0xF], absmax[(j + 1) / blocksize]);
        res[4 * w + b] = pack_bf16x2(hi, lo);
      }
    }
    out[2 * gi] = make_uint4(res[0], res[1], res[2], res[3]);
    out[2 * gi + 1] = make_uint4(res[4], res[5], res[6], res[7]);
  }
}

__global__ void nf4_dequant_tail(const uint8_t* __restrict__ packed, const float* __restrict__ absmax, int blocksize,
                                 int64_t first_byte, int64_t bytes, __nv_bfloat16* __restrict__ out) {
  const int64_t b = first_byte + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b >= bytes) return;
  const uint8_t v = packed[b];
  out[2 * b] = __float2bfloat16_rn(__fmul_rn(kNF4Levels[v >> 4], absmax[(2 * b) / blocksize]));
  out[2 * b + 1] = __float2bfloat16_rn(__fmul_rn(kNF4Levels[v & 0xF], absmax[(2 * b + 1) / blocksize]));
}

// out[e][g][r] (experts, cols/64, rows): NF4 the absmax of block (e, r, g) (storage order), else the bf16 value of
// the block scale covering group g of row r.
__global__ void quant_multipliers(int nf4, const float* __restrict__ src, int64_t rows, int64_t groups, int sr, int sc,
                                  int64_t br, int64_t bc, int64_t total, float* __restrict__ out) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t per = groups * rows;
    const int64_t e = i / per, rem = i - e * per;
    const int64_t g = rem / rows, r = rem - g * rows;
    out[i] = nf4 ? src[(e * rows + r) * groups + g]
                 : bf16_round(src[(e * sr + r / br) * sc + (64 * g) / bc]);
  }
}

// Vector forms of the three dequantisations: 16 weights per thread step (16 code bytes or 8 NF4 bytes in, 32 bytes
// out), one scale or absmax look-up and one index computation per 16 weights. They apply when every group of 16
// lies in one expert / block / 64-weight NF4 block (the launchers check), otherwise the element kernels above run.

// bf16(f32(w8) * scale[e]) for 16 codes of expert e (per_expert a multiple of 16).
__global__ void stack_dequant16(const uint4* __restrict__ codes, const float* __restrict__ scale, int64_t per16,
                                int64_t groups, uint4* __restrict__ out) {
  for (int64_t gi = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; gi < groups;
       gi += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint4 c = codes[gi];
    const float s = scale[gi / per16];
    const uint32_t w[4] = {c.x, c.y, c.z, c.w};
    uint32_t o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const __nv_bfloat162 v = e4m3x2_to_bf16x2(w[j >> 1], (j & 1) ? 0x3424u : 0x1404u);  // exact
      const uint32_t b = *reinterpret_cast<const uint32_t*>(&v);
      o[j] = pack_bf16x2(__fmul_rn(bf16_lo(b), s), __fmul_rn(bf16_hi(b), s));
    }
    out[2 * gi] = make_uint4(o[0], o[1], o[2], o[3]);
    out[2 * gi + 1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

// bf16(bf16(w8) * bf16(s)) for 16 codes of one row within one block (cols and the block width multiples of 16):
// the product of the exact bf16 code and the bf16 scale is exact before its one rounding, so a bf16x2 multiply gives
// the same bits as the float32 multiply and conversion.
__global__ void block_dequant16(const uint4* __restrict__ codes, int64_t rows, int64_t cols16,
                                const float* __restrict__ scale_inv, int sr, int sc, int64_t br, int64_t bc,
                                int64_t groups, uint4* __restrict__ out) {
  for (int64_t gi = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; gi < groups;
       gi += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t rowi = gi / cols16, c = (gi - rowi * cols16) * 16;
    const int64_t m = rowi / rows, r = rowi - m * rows;
    const float s = bf16_round(scale_inv[(m * sr + r / br) * sc + c / bc]);
    const __nv_bfloat162 s2 = __float2bfloat162_rn(s);
    const uint4 cw = codes[gi];
    const uint32_t w[4] = {cw.x, cw.y, cw.z, cw.w};
    uint32_t o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const __nv_bfloat162 v = __hmul2(e4m3x2_to_bf16x2(w[j >> 1], (j & 1) ? 0x3424u : 0x1404u), s2);
      o[j] = *reinterpret_cast<const uint32_t*>(&v);
    }
    out[2 * gi] = make_uint4(o[0], o[1], o[2], o[3]);
    out[2 * gi + 1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

// NF4, 16 weights (8 bytes) per step within one block of `blocksize` (a multiple of 16): the levels from shared
// memory (constant memory serialises divergent reads), one absmax per 16 weights.
__global__ void nf4_dequant16(const uint2* __restrict__ packed, const float* __restrict__ absmax, int64_t per_block16,
                              int64_t groups, uint4* __restrict__ out) {
  __shared__ float lv[16];
  if (threadIdx.x < 16) lv[threadIdx.x] = kNF4Levels[threadIdx.x];
  __syncthreads();
  for (int64_t gi = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; gi < groups;
       gi += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint2 p = packed[gi];
    const float a = absmax[gi / per_block16];
    const uint32_t words[2] = {p.x, p.y};
    uint32_t res[8];
#pragma unroll
    for (int w = 0; w < 2; ++w) {
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t byte = (words[w] >> (8 * b)) & 0xFF;
        res[4 * w + b] = pack_bf16x2(__fmul_rn(lv[byte >> 4], a), __fmul_rn(lv[byte & 0xF], a));
      }
    }
    out[2 * gi] = make_uint4(res[0], res[1], res[2], res[3]);
    out[2 * gi + 1] = make_uint4(res[4], res[5], res[6], res[7]);
  }
}

inline unsigned grid_for(int64_t n, int threads = 256) {
  int64_t b = (n + threads - 1) / threads;
  if (b > 148 * 32) b = 148 * 32;
  return static_cast<unsigned>(b > 0 ? b : 1);
}

}  // namespace quant
}  // namespace meep2b

using namespace meep2b;
using namespace meep2b::quant;

extern "C" {

int meep2b_fp8_stack_quantize(const void* w, int32_t dtype, int32_t experts, int64_t per_expert, uint8_t* codes,
                              float* scale, float* workspace, void* stream) {
  if (experts < 1 || per_expert < 1) return MEEP2B_ERR_SHAPE;
  if (dtype != MEEP2B_F32 && dtype != MEEP2B_BF16) return MEEP2B_ERR_DTYPE;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  cudaMemsetAsync(workspace, 0, sizeof(float) * experts, s);
  int64_t bx = (per_expert + 255) / 256;
  if (bx > 256) bx = 256;
  dim3 grid(static_cast<unsigned>(bx), static_cast<unsigned>(experts));
  if (dtype == MEEP2B_BF16) {
    stack_amax<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(w), per_expert, workspace);
    stack_cast<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(w), per_expert, workspace,
                                                   codes, scale);
  } else {
    stack_amax<float><<<grid, 256, 0, s>>>(static_cast<const float*>(w), per_expert, workspace);
    stack_cast<float><<<grid, 256, 0, s>>>(static_cast<const float*>(w), per_expert, workspace, codes, scale);
  }
  return launch_status();
}

int meep2b_fp8_stack_dequantize(const uint8_t* codes, const float* scale, int32_t experts, int64_t per_expert,
                                void* out, void* stream) {
  if (experts < 1 || per_expert < 1) return MEEP2B_ERR_SHAPE;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  const int64_t total = per_expert * experts;
  if (per_expert % 16 == 0 && aligned16(codes) && aligned16(out)) {
    stack_dequant16<<<grid_for(total / 16), 256, 0, s>>>(reinterpret_cast<const uint4*>(codes), scale, per_expert / 16,
                                                         total / 16, static_cast<uint4*>(out));
  } else {
    stack_dequant<<<grid_for(total), 256, 0, s>>>(codes, scale, per_expert, total, static_cast<__nv_bfloat16*>(out));
  }
  return launch_status();
}

int meep2b_fp8_block_dequantize(const uint8_t* codes, int64_t matrices, int64_t rows, int64_t cols,
                                const float* scale_inv, int32_t sr, int32_t sc, void* out, void* stream) {
  if (matrices < 1 || rows < 1 || cols < 1 || sr < 1 || sc < 1) return MEEP2B_ERR_SHAPE;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  const int64_t br = (rows + sr - 1) / sr, bc = (cols + sc - 1) / sc;
  const int64_t total = matrices * rows * cols;
  if (cols % 16 == 0 && bc % 16 == 0 && aligned16(codes) && aligned16(out)) {
    block_dequant16<<<grid_for(total / 16), 256, 0, s>>>(reinterpret_cast<const uint4*>(codes), rows, cols / 16,
                                                         scale_inv, sr, sc, br, bc, total / 16,
                                                         static_cast<uint4*>(out));
  } else {
    block_dequant<<<grid_for(total), 256, 0, s>>>(codes, rows, cols, scale_inv, sr, sc, br, bc, total,
                                                  static_cast<__nv_bfloat16*>(out));
  }
  return launch_status();
}

int meep2b_fp8_block_quantize(const void* w, int32_t dtype, int64_t matrices, int64_t rows, int64_t cols, int32_t sr,
                              int32_t sc, uint8_t* codes, float* scale_inv, void* stream) {
  if (matrices < 1 || rows < 1 || cols < 1 || sr < 1 || sc < 1 || matrices > 65535) return MEEP2B_ERR_SHAPE;
  if (dtype != MEEP2B_F32 && dtype != MEEP2B_BF16) return MEEP2B_ERR_DTYPE;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  const int64_t br = (rows + sr - 1) / sr, bc = (cols + sc - 1) / sc;
  dim3 grid(static_cast<unsigned>(sc), static_cast<unsigned>(sr), static_cast<unsigned>(matrices));
  if (dtype == MEEP2B_BF16)
    block_quant<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(w), rows, cols, sr, sc, br, bc,
                                                    codes, scale_inv);
  else
    block_quant<float><<<grid, 256, 0, s>>>(static_cast<const float*>(w), rows, cols, sr, sc, br, bc, codes,
                                            scale_inv);
  return launch_status();
}

int meep2b_quant_multipliers(int32_t weight_dtype, const float* src, int32_t experts, int64_t rows, int64_t cols,
                             int32_t sr, int32_t sc, float* out, void* stream) {
  if (experts < 1 || rows < 1 || cols < 64 || cols % 64) return MEEP2B_ERR_SHAPE;
  if (weight_dtype != MEEP2B_NF4 && weight_dtype != MEEP2B_E4M3_BLOCKS) return MEEP2B_ERR_DTYPE;
  int64_t br = 1, bc = 64;
  if (weight_dtype == MEEP2B_E4M3_BLOCKS) {
    if (sr < 1 || sc < 1 || sr > rows || sc > cols) return MEEP2B_ERR_SHAPE;
    br = (rows + sr - 1) / sr;
    bc = (cols + sc - 1) / sc;
    if (bc % 64) return MEEP2B_ERR_UNSUPPORTED;
  }
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  const int64_t total = static_cast<int64_t>(experts) * rows * (cols / 64);
  quant_multipliers<<<grid_for(total), 256, 0, s>>>(weight_dtype == MEEP2B_NF4, src, rows, cols / 64, sr, sc, br, bc,
                                                     total, out);
  return launch_status();
}

int meep2b_nf4_absmax(const uint8_t* absmax, const float* absmax2, const float* code2, const float* offset,
                      int32_t blocksize2, int64_t count, float* absmax_out, void* stream) {
  if (count < 1 || blocksize2 < 1) return MEEP2B_ERR_SHAPE;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  nf4_absmax<<<grid_for(count), 256, 0, s>>>(absmax, absmax2, code2, offset, blocksize2, count, absmax_out);
  return launch_status();
}

int meep2b_nf4_dequantize(const uint8_t* packed, const uint8_t* absmax, const float* absmax2, const float* code2,
                          const float* offset, int32_t blocksize, int32_t blocksize2, int64_t n, float* absmax_out,
                          void* out, void* stream) {
  if (n < 2 || n % 2 || blocksize < 2 || blocksize2 < 1) return MEEP2B_ERR_SHAPE;
  if (!aligned16(out) || (reinterpret_cast<uintptr_t>(packed) & 7)) return MEEP2B_ERR_ALIGN;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  const int64_t blocks = (n + blocksize - 1) / blocksize;
  nf4_absmax<<<grid_for(blocks), 256, 0, s>>>(absmax, absmax2, code2, offset, blocksize2, blocks, absmax_out);
  const int64_t bytes = n / 2;
  const int64_t groups = bytes / 8;
  if (groups > 0 && blocksize % 16 == 0) {
    nf4_dequant16<<<grid_for(groups), 256, 0, s>>>(reinterpret_cast<const uint2*>(packed), absmax_out,
                                                   blocksize / 16, groups, static_cast<uint4*>(out));
  } else if (groups > 0) {
    nf4_dequant<<<grid_for(groups), 256, 0, s>>>(reinterpret_cast<const uint2*>(packed), absmax_out, blocksize, groups,
                                                 static_cast<uint4*>(out));
  }
  if (groups * 8 < bytes)
    nf4_dequant_tail<<<1, 256, 0, s>>>(packed, absmax_out, blocksize, groups * 8, bytes,
                                       static_cast<__nv_bfloat16*>(out));
  return launch_status();
}

}  // extern "C"

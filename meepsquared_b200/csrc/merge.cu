// The merged save of an expert stack (meepsquared/_save.py:79-95, `_merged_stack`): every expert's frozen weight,
// dequantised to float32, plus its adapter's update, out = dtype(W_e + scaling * (lhs_e @ rhs_e)), in the stack's
// own layout (lhs_e @ rhs_e is (rows, cols) like W_e). An FP8 stack with one scale per expert is dequantised as
// _fp8.dequantize_stack does for float32 (f32(code) * scale[e], one rounding). Elementwise over the stack and
// HBM-bound (the weight read once, the merged weight written once); the factors, rank x 256 columns of rhs per
// block (for 256 rows) and 32 rows x rank of lhs per row tile, are staged in shared memory; each thread makes 4
// rows by two runs of 4 columns,
// summing the rank products in order j = 0 .. rank - 1 with fused multiply-adds. Included after quant.cu (its exact
// e4m3 conversion).
#include "common.cuh"
#include "host.hpp"

namespace meep2b {
namespace merge {

constexpr int MROWS = 32;   // rows of a block's tile
constexpr int MCOLS = 256;  // columns of a block's tile
constexpr int MTILES = 8;   // row tiles per block: the staged columns of rhs serve 256 rows
constexpr int MAX_RANK = 128;

// A thread's columns of a row tile: two runs of 4, at 4 lane and 128 + 4 lane of the block's 256 (so that a warp's
// shared-memory reads of rhs and its global accesses are each one contiguous run).
template <int WT>
__device__ __forceinline__ void load_run(const void* weight, int64_t at, uint4& raw) {
  if (WT == MEEP2B_E4M3) {
    raw.x = *reinterpret_cast<const uint32_t*>(static_cast<const uint8_t*>(weight) + at);
  } else if (WT == MEEP2B_BF16) {
    const uint2 q = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(weight) + at);
    raw.x = q.x, raw.y = q.y;
  } else {
    raw = *reinterpret_cast<const uint4*>(static_cast<const float*>(weight) + at);
  }
}

template <int WT>
__device__ __forceinline__ float weight_at(const void* weight, int64_t at, float se) {
  if (WT == MEEP2B_E4M3) return __fmul_rn(quant::e4m3_to_float(static_cast<const uint8_t*>(weight)[at]), se);
  if (WT == MEEP2B_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(weight)[at]);
  return static_cast<const float*>(weight)[at];
}

template <int WT>
__device__ __forceinline__ void decode_run(const uint4& raw, float se, float* w) {
  if (WT == MEEP2B_E4M3) {
#pragma unroll
    for (int b = 0; b < 4; ++b) w[b] = __fmul_rn(quant::e4m3_to_float(static_cast<uint8_t>(raw.x >> (8 * b))), se);
  } else if (WT == MEEP2B_BF16) {
    w[0] = bf16_lo(raw.x), w[1] = bf16_hi(raw.x), w[2] = bf16_lo(raw.y), w[3] = bf16_hi(raw.y);
  } else {
    w[0] = __uint_as_float(raw.x), w[1] = __uint_as_float(raw.y), w[2] = __uint_as_float(raw.z);
    w[3] = __uint_as_float(raw.w);
  }
}

template <int OT>
__device__ __forceinline__ void store_run(void* out, int64_t at, const float* v) {
  if (OT == MEEP2B_BF16) {
    *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(out) + at) =
        make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
  } else {
    *reinterpret_cast<float4*>(static_cast<float*>(out) + at) = make_float4(v[0], v[1], v[2], v[3]);
  }
}

template <int WT, int OT>
__global__ void __launch_bounds__(256) merge_stack_kernel(const void* __restrict__ weight,
                                                          const float* __restrict__ scale,
                                                          const float* __restrict__ lhs,
                                                          const float* __restrict__ rhs, int rank, float scaling,
                                                          int64_t rows, int64_t cols, void* __restrict__ out) {
  extern __shared__ float sm[];
  const int rank4 = (rank + 3) & ~3;
  float* rhs_s = sm;                  // [rank][MCOLS]
  float* lhs_s = sm + rank * MCOLS;   // [MROWS][rank4], zero past rank
  const int64_t e = blockIdx.z;
  const int64_t r_block = static_cast<int64_t>(blockIdx.y) * MROWS * MTILES;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * MCOLS;
  const float* rhs_e = rhs + e * rank * cols;
  const float* lhs_e = lhs + e * rows * rank;
  for (int i = threadIdx.x; i < rank * MCOLS; i += blockDim.x) {
    const int j = i / MCOLS, c = i - j * MCOLS;
    rhs_s[i] = c0 + c < cols ? rhs_e[j * cols + c0 + c] : 0.0f;
  }
  const int tr = (threadIdx.x >> 5) * 4;  // this thread's 4 rows of a row tile
  const int lane = threadIdx.x & 31;
  const int64_t col[2] = {c0 + 4 * lane, c0 + 128 + 4 * lane};  // its two runs of 4 columns
  const bool vec = (cols & 3) == 0;  // whole runs: 4-, 8- or 16-byte accesses
  const float se = WT == MEEP2B_E4M3 ? scale[e] : 1.0f;
  for (int rt = 0; rt < MTILES; ++rt) {  // the block's row tiles, all with the staged columns of rhs
    const int64_t r0 = r_block + static_cast<int64_t>(rt) * MROWS;
    if (r0 >= rows) break;
    // this thread's weights first: their loads are in flight while the rank products are summed
    uint4 raw[4][2];
#pragma unroll
    for (int a = 0; a < 4; ++a) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        raw[a][h] = make_uint4(0u, 0u, 0u, 0u);
        const int64_t r = r0 + tr + a;
        if (vec && r < rows && col[h] < cols) load_run<WT>(weight, (e * rows + r) * cols + col[h], raw[a][h]);
      }
    }
    __syncthreads();  // rhs staged; the previous row tile's reads of lhs_s are done
    for (int i = threadIdx.x; i < MROWS * rank4; i += blockDim.x) {
      const int rr = i / rank4, j = i - rr * rank4;
      lhs_s[i] = r0 + rr < rows && j < rank ? lhs_e[(r0 + rr) * rank + j] : 0.0f;
    }
    __syncthreads();
    float acc[4][8];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 8; ++b) acc[a][b] = 0.0f;
    for (int j4 = 0; j4 < rank; j4 += 4) {
      float4 l4[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) l4[a] = *reinterpret_cast<const float4*>(lhs_s + (tr + a) * rank4 + j4);
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int j = j4 + jj;
        if (j >= rank) break;  // rows of rhs past rank are not staged
        const float4 q0 = *reinterpret_cast<const float4*>(rhs_s + j * MCOLS + 4 * lane);
        const float4 q1 = *reinterpret_cast<const float4*>(rhs_s + j * MCOLS + 128 + 4 * lane);
        const float q[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          const float l = jj == 0 ? l4[a].x : jj == 1 ? l4[a].y : jj == 2 ? l4[a].z : l4[a].w;
#pragma unroll
          for (int b = 0; b < 8; ++b) acc[a][b] = __fmaf_rn(l, q[b], acc[a][b]);
        }
      }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const int64_t r = r0 + tr + a;
      if (r >= rows) break;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (col[h] >= cols) continue;
        const int64_t at = (e * rows + r) * cols + col[h];
        float w[4], v[4];
        if (vec) {
          decode_run<WT>(raw[a][h], se, w);
        } else {
#pragma unroll
          for (int b = 0; b < 4; ++b) w[b] = col[h] + b < cols ? weight_at<WT>(weight, at + b, se) : 0.0f;
        }
#pragma unroll
        for (int b = 0; b < 4; ++b) v[b] = rank > 0 ? __fadd_rn(w[b], __fmul_rn(scaling, acc[a][4 * h + b])) : w[b];
        if (vec) {
          store_run<OT>(out, at, v);
        } else {
          for (int b = 0; b < 4 && col[h] + b < cols; ++b) {
            if (OT == MEEP2B_BF16) {
              static_cast<__nv_bfloat16*>(out)[at + b] = __float2bfloat16_rn(v[b]);
            } else {
              static_cast<float*>(out)[at + b] = v[b];
            }
          }
        }
      }
    }
  }
}

template <int WT, int OT>
static int launch_merge(const void* weight, const float* scale, const float* lhs, const float* rhs, int rank,
                        float scaling, int64_t experts, int64_t rows, int64_t cols, void* out, cudaStream_t s) {
  const size_t rank4 = static_cast<size_t>((rank + 3) & ~3);
  const size_t smem = sizeof(float) * (static_cast<size_t>(rank) * MCOLS + rank4 * MROWS + 4);
  auto kern = merge_stack_kernel<WT, OT>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess) {
    cudaGetLastError();
    return MEEP2B_ERR_LAUNCH;
  }
  const int64_t row_blocks = (rows + MROWS * MTILES - 1) / (MROWS * MTILES);
  const dim3 grid(static_cast<unsigned>((cols + MCOLS - 1) / MCOLS), static_cast<unsigned>(row_blocks),
                  static_cast<unsigned>(experts));
  kern<<<grid, 256, smem, s>>>(weight, scale, lhs, rhs, rank, scaling, rows, cols, out);
  return launch_status();
}

}  // namespace merge
}  // namespace meep2b

using namespace meep2b;

extern "C" int meep2b_merge_stack(const void* weight, int32_t weight_dtype, const float* scale, const float* lhs,
                                  const float* rhs, int32_t rank, float scaling, int64_t experts, int64_t rows,
                                  int64_t cols, void* out, int32_t out_dtype, void* stream) {
  if (experts < 0 || rows < 0 || cols < 0 || rank < 0 || rank > merge::MAX_RANK) return MEEP2B_ERR_SHAPE;
  if (experts > 65535 || (rows + merge::MROWS - 1) / merge::MROWS > 65535) return MEEP2B_ERR_SHAPE;
  if (weight_dtype != MEEP2B_F32 && weight_dtype != MEEP2B_BF16 && weight_dtype != MEEP2B_E4M3) return MEEP2B_ERR_DTYPE;
  if (out_dtype != MEEP2B_F32 && out_dtype != MEEP2B_BF16) return MEEP2B_ERR_DTYPE;
  if (weight_dtype == MEEP2B_E4M3 && scale == nullptr) return MEEP2B_ERR_SHAPE;
  if (rank > 0 && (lhs == nullptr || rhs == nullptr)) return MEEP2B_ERR_SHAPE;
  if (!aligned16(lhs) || !aligned16(rhs) || !aligned16(weight) || !aligned16(out)) return MEEP2B_ERR_ALIGN;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  if (experts == 0 || rows == 0 || cols == 0) return MEEP2B_OK;
#define MEEP2B_MERGE(W, O) \
  merge::launch_merge<W, O>(weight, scale, lhs, rhs, rank, scaling, experts, rows, cols, out, s)
  if (out_dtype == MEEP2B_BF16) {
    if (weight_dtype == MEEP2B_E4M3) return MEEP2B_MERGE(MEEP2B_E4M3, MEEP2B_BF16);
    if (weight_dtype == MEEP2B_BF16) return MEEP2B_MERGE(MEEP2B_BF16, MEEP2B_BF16);
    return MEEP2B_MERGE(MEEP2B_F32, MEEP2B_BF16);
  }
  if (weight_dtype == MEEP2B_E4M3) return MEEP2B_MERGE(MEEP2B_E4M3, MEEP2B_F32);
  if (weight_dtype == MEEP2B_BF16) return MEEP2B_MERGE(MEEP2B_BF16, MEEP2B_F32);
  return MEEP2B_MERGE(MEEP2B_F32, MEEP2B_F32);
#undef MEEP2B_MERGE
}

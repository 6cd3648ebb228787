// The adapters' gradients: out[e, j, r] = bf16(s * sum over expert e's rows of g[row, j] * low[row, r]), r < 16.
//
// Replaces _grouped_reduce_kernel / _reduce (meepsquared/_grouped.py:233-256, 362-370). This is a streaming
// reduction over each expert's rows with an output of only (n x 16) per expert: it reads g once (the dominant
// traffic) and is bound by HBM bandwidth, not by tensor throughput (16 MACs per element of g). The small
// products run on the warp-level mma.sync m16n8k16 path, fed from shared memory by ldmatrix.trans: the operand
// tiles are row-major in memory and the MMA wants them transposed. Rows stream through a two-stage cp.async
// ring of 64-row chunks.
//
// Grid: (ceil(n / 128), experts); 8 warps, warp w owns columns [16 w, 16 w + 16) of the CTA's 128.
// The gathered form reads row i of g as g[g_rows[i]] (the routed rows straight from the token-major tensor, no
// expert-sorted copy) and weights it by row_scale[i]; the weight is applied to the rank panel's row
// (bf16(row_scale * low), 16 values) rather than to the n values of g.
#include "common.cuh"
#include "host.hpp"

namespace meep2b {
namespace reduce {

constexpr int COLS = 128;
constexpr int ROWS = 64;
constexpr int G_PITCH = COLS + 8;   // bf16 elements per smem row of g: 272 bytes, no ldmatrix bank conflicts
constexpr int L_PITCH = 16 + 8;     // of low: 48 bytes
constexpr int THREADS = 256;

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool pred) {
  const uint32_t d = smem_u32(dst);
  const int bytes = pred ? 16 : 0;  // zero-fill when out of range
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(THREADS) grouped_reduce_kernel(const __nv_bfloat16* __restrict__ g, int64_t n,
                                                                 int64_t ldg, const __nv_bfloat16* __restrict__ low,
                                                                 const int32_t* __restrict__ offsets, float scaling,
                                                                 __nv_bfloat16* __restrict__ out,
                                                                 const int32_t* __restrict__ g_rows,
                                                                 const float* __restrict__ row_scale) {
  __shared__ __align__(16) __nv_bfloat16 gs[2][ROWS][G_PITCH];
  __shared__ __align__(16) __nv_bfloat16 ls[2][ROWS][L_PITCH];
  const int e = blockIdx.y;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * COLS;
  const int64_t start = e > 0 ? offsets[e - 1] : 0;
  const int64_t end = offsets[e];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  float acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};  // [n-tile of 8 ranks][fragment]
  const int chunks = static_cast<int>((end - start + ROWS - 1) / ROWS);

  auto load = [&](int chunk, int buf) {
    const int64_t r0 = start + static_cast<int64_t>(chunk) * ROWS;
    // g: 64 rows x 128 columns = 1024 16-byte pieces, 4 per thread
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int piece = threadIdx.x + i * THREADS;
      const int r = piece >> 4, c = (piece & 15) * 8;
      const int64_t row = r0 + r, col = c0 + c;
      const bool ok = row < end && col < n;
      const int64_t src = ok && g_rows != nullptr ? static_cast<int64_t>(g_rows[row]) : row;
      cp_async16(&gs[buf][r][c], ok ? g + src * ldg + col : g, ok);
    }
    // low: 64 rows x 16 = 128 pieces
    if (threadIdx.x < 128) {
      const int r = threadIdx.x >> 1, c = (threadIdx.x & 1) * 8;
      const int64_t row = r0 + r;
      const bool ok = row < end;
      if (row_scale == nullptr) {
        cp_async16(&ls[buf][r][c], ok ? low + row * 16 + c : low, ok);
      } else {  // bf16(w * low): a plain load, scaled and stored (the ring's barrier also covers these stores)
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (ok) {
          const uint4 l = *reinterpret_cast<const uint4*>(low + row * 16 + c);
          const float w = row_scale[row];
          const uint32_t in[4] = {l.x, l.y, l.z, l.w};
          uint32_t o[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) o[j] = pack_bf16x2(bf16_lo(in[j]) * w, bf16_hi(in[j]) * w);
          v = make_uint4(o[0], o[1], o[2], o[3]);
        }
        *reinterpret_cast<uint4*>(&ls[buf][r][c]) = v;
      }
    }
    cp_async_commit();
  };

  if (chunks > 0) load(0, 0);
  for (int ch = 0; ch < chunks; ++ch) {
    const int buf = ch & 1;
    if (ch + 1 < chunks) {
      load(ch + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < ROWS / 16; ++kk) {
      // A (16 columns x 16 rows) = g^T: the four 8x8 blocks (cols 0-7|8-15) x (rows 0-7|8-15), transposed
      uint32_t a[4];
      {
        const int mtx = lane >> 3, r = lane & 7;
        const int row = kk * 16 + (mtx >> 1) * 8 + r;
        const int col = warp * 16 + (mtx & 1) * 8;
        ldmatrix_x4_trans(a, &gs[buf][row][col]);
      }
      // B (16 rows x 16 ranks) = low: blocks (rows 0-7|8-15) x (ranks 0-7|8-15), transposed
      uint32_t b[4];
      {
        const int mtx = lane >> 3, r = lane & 7;
        const int row = kk * 16 + (mtx & 1) * 8 + r;
        const int col = (mtx >> 1) * 8;
        ldmatrix_x4_trans(b, &ls[buf][row][col]);
      }
      mma16816(acc[0], a, b[0], b[1]);
      mma16816(acc[1], a, b[2], b[3]);
    }
    __syncthreads();
  }
  // C fragment: c0,c1 -> (column = lane/4, ranks 2(lane%4)+{0,1}); c2,c3 -> column + 8
  const int64_t col_a = c0 + warp * 16 + (lane >> 2);
  __nv_bfloat16* o = out + static_cast<int64_t>(e) * n * 16;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    const int rk = nt * 8 + 2 * (lane & 3);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t col = col_a + h * 8;
      if (col < n) {
        const uint32_t v = pack_bf16x2(acc[nt][2 * h] * scaling, acc[nt][2 * h + 1] * scaling);
        *reinterpret_cast<uint32_t*>(o + col * 16 + rk) = v;
      }
    }
  }
}

}  // namespace reduce
}  // namespace meep2b

static int grouped_reduce_launch(const void* g, const int32_t* g_rows, const float* row_scale, int64_t rows,
                                 int64_t n, int64_t ldg, const void* low, const int32_t* offsets, int32_t experts,
                                 float scaling, void* out, void* stream) {
  using namespace meep2b;
  if (rows < 0 || n < 1 || experts < 1 || ldg < n) return MEEP2B_ERR_SHAPE;
  if (n % 8 || ldg % 8) return MEEP2B_ERR_ALIGN;
  if (!aligned16(g) || !aligned16(low) || !aligned16(out)) return MEEP2B_ERR_ALIGN;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  dim3 grid(static_cast<unsigned>((n + reduce::COLS - 1) / reduce::COLS), static_cast<unsigned>(experts));
  reduce::grouped_reduce_kernel<<<grid, reduce::THREADS, 0, s>>>(
      static_cast<const __nv_bfloat16*>(g), n, ldg, static_cast<const __nv_bfloat16*>(low), offsets, scaling,
      static_cast<__nv_bfloat16*>(out), g_rows, row_scale);
  return launch_status();
}

extern "C" int meep2b_grouped_reduce(const void* g, int64_t rows, int64_t n, int64_t ldg, const void* low,
                                     const int32_t* offsets, int32_t experts, float scaling, void* out,
                                     void* stream) {
  return grouped_reduce_launch(g, nullptr, nullptr, rows, n, ldg, low, offsets, experts, scaling, out, stream);
}

extern "C" int meep2b_grouped_reduce_rows(const void* g, const int32_t* g_rows, const float* row_scale,
                                          int64_t rows, int64_t n, int64_t ldg, const void* low,
                                          const int32_t* offsets, int32_t experts, float scaling, void* out,
                                          void* stream) {
  if (g_rows == nullptr) return MEEP2B_ERR_SHAPE;
  return grouped_reduce_launch(g, g_rows, row_scale, rows, n, ldg, low, offsets, experts, scaling, out, stream);
}

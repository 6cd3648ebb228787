// The adapters' gradients: out[e, j, r] = bf16(s * sum over expert e's rows of g[row, j] * low[row, r]), r < 16.
//
// Replaces _grouped_reduce_kernel / _reduce (meepsquared/_grouped.py:233-256, 362-370). This is a streaming
// reduction over each expert's rows with an output of only (n x 16) per expert: it reads g once (the dominant
// traffic) and is bound by HBM bandwidth, not by tensor throughput (16 MACs per element of g). The small
// products run on the warp-level mma.sync m16n8k16 path, fed from shared memory by ldmatrix.trans: the operand
// tiles are row-major in memory and the MMA wants them transposed. Rows stream through a two-stage cp.async
// ring of 64-row chunks; nothing waits on a plain load inside the loop (the gathered form's row indices are read a
// chunk ahead, the row weights come in by cp.async with the panel and are applied in shared memory).
//
// Grid: (ceil(n / COLS), experts); COLS / 16 warps, warp w owns columns [16 w, 16 w + 16) of the CTA's COLS
// (128: 8 warps; the kernel also builds for 64).
// The gathered form reads row i of g as g[g_rows[i]] (the routed rows straight from the token-major tensor, no
// expert-sorted copy) and weights it by row_scale[i]; the weight is applied to the rank panel's row
// (bf16(row_scale * low), 16 values) rather than to the n values of g.
#include "common.cuh"
#include "host.hpp"

namespace meep2b {
namespace reduce {

constexpr int ROWS = 64;
constexpr int L_PITCH = 16 + 8;     // of low: 48 bytes

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

__device__ __forceinline__ void cp_async4(void* dst, const void* src, bool pred) {
  const uint32_t d = smem_u32(dst);
  const int bytes = pred ? 4 : 0;
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(d), "l"(src), "r"(bytes) : "memory");
}

template <int COLS>
__global__ void __launch_bounds__(COLS * 2) grouped_reduce_kernel(const __nv_bfloat16* __restrict__ g, int64_t n,
                                                                 int64_t ldg, const __nv_bfloat16* __restrict__ low,
                                                                 const int32_t* __restrict__ offsets, float scaling,
                                                                 __nv_bfloat16* __restrict__ out,
                                                                 const int32_t* __restrict__ g_rows,
                                                                 const float* __restrict__ row_scale,
                                                                 int out_layout) {
  constexpr int THREADS = COLS * 2;
  constexpr int G_PITCH = COLS + 8;  // bf16 elements per smem row of g (+16 bytes: no ldmatrix bank conflicts)
  constexpr int PIECES_PER_ROW = COLS / 8;
  constexpr int ROWS_PER_PASS = THREADS / PIECES_PER_ROW;  // 16
  __shared__ __align__(16) __nv_bfloat16 gs[2][ROWS][G_PITCH];
  __shared__ __align__(16) __nv_bfloat16 ls[2][ROWS][L_PITCH];
  __shared__ float ws[2][ROWS];
  const int e = blockIdx.y;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * COLS;
  const int64_t start = e > 0 ? offsets[e - 1] : 0;
  const int64_t end = offsets[e];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  float acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};  // [n-tile of 8 ranks][fragment]
  const int chunks = static_cast<int>((end - start + ROWS - 1) / ROWS);

  // This thread's four g pieces of a chunk are rows piece_row + 16 i (i < 4) at column piece_col. The source rows of
  // gathered g are read one chunk ahead of their copies, so that no copy waits for its index.
  const int piece_row = threadIdx.x / PIECES_PER_ROW, piece_col = (threadIdx.x % PIECES_PER_ROW) * 8;
  static_assert(ROWS_PER_PASS * 4 == ROWS, "four passes of 16-byte pieces cover a chunk");
  auto sources = [&](int chunk, int64_t (&src)[4]) {
    const int64_t r0 = start + static_cast<int64_t>(chunk) * ROWS;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t row = r0 + piece_row + ROWS_PER_PASS * i;
      src[i] = row < end ? (g_rows != nullptr ? static_cast<int64_t>(__ldg(g_rows + row)) : row) : -1;
    }
  };
  auto load = [&](int chunk, int buf, const int64_t (&src)[4]) {
    const int64_t r0 = start + static_cast<int64_t>(chunk) * ROWS;
    // g: 64 rows x COLS columns of 16-byte pieces, 4 per thread
    const int64_t col = c0 + piece_col;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const bool ok = src[i] >= 0 && col < n;
      cp_async16(&gs[buf][piece_row + ROWS_PER_PASS * i][piece_col], ok ? g + src[i] * ldg + col : g, ok);
    }
    // low: 64 rows x 16 = 128 pieces; the rows' weights (row-scaled form), one float each
    for (int i = threadIdx.x; i < 128; i += THREADS) {
      const int r = i >> 1, c = (i & 1) * 8;
      const int64_t row = r0 + r;
      const bool ok = row < end;
      cp_async16(&ls[buf][r][c], ok ? low + row * 16 + c : low, ok);
    }
    if (row_scale != nullptr) {
      const int r = THREADS >= 128 + ROWS ? static_cast<int>(threadIdx.x) - 128 : static_cast<int>(threadIdx.x);
      if (r >= 0 && r < ROWS) {
        const int64_t row = r0 + r;
        cp_async4(&ws[buf][r], row < end ? row_scale + row : row_scale, row < end);
      }
    }
    cp_async_commit();
  };

  int64_t src_next[4];
  if (chunks > 0) {
    int64_t src0[4];
    sources(0, src0);
    load(0, 0, src0);
  }
  if (chunks > 1) sources(1, src_next);
  for (int ch = 0; ch < chunks; ++ch) {
    const int buf = ch & 1;
    if (ch + 1 < chunks) {
      load(ch + 1, buf ^ 1, src_next);
      if (ch + 2 < chunks) sources(ch + 2, src_next);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (row_scale != nullptr) {  // bf16(w * low) in place: 1024 values, 4 at a time
      for (int i = threadIdx.x; i < ROWS * 4; i += THREADS) {
        const int r = i >> 2, c = (i & 3) * 4;
        const float w = ws[buf][r];
        uint2* p2 = reinterpret_cast<uint2*>(&ls[buf][r][c]);
        const uint2 v = *p2;
        *p2 = make_uint2(pack_bf16x2(bf16_lo(v.x) * w, bf16_hi(v.x) * w),
                         pack_bf16x2(bf16_lo(v.y) * w, bf16_hi(v.y) * w));
      }
      __syncthreads();
    }
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
        if (out_layout == 0) {
          *reinterpret_cast<uint32_t*>(o + col * 16 + rk) = v;
        } else {  // (16, n) per expert
          o[rk * n + col] = __ushort_as_bfloat16(static_cast<unsigned short>(v & 0xFFFFu));
          o[(rk + 1) * n + col] = __ushort_as_bfloat16(static_cast<unsigned short>(v >> 16));
        }
      }
    }
  }
}

}  // namespace reduce
}  // namespace meep2b

static int grouped_reduce_launch(const void* g, const int32_t* g_rows, const float* row_scale, int64_t rows,
                                 int64_t n, int64_t ldg, const void* low, const int32_t* offsets, int32_t experts,
                                 float scaling, void* out, int32_t out_layout, void* stream) {
  using namespace meep2b;
  if (rows < 0 || n < 1 || experts < 1 || ldg < n || out_layout < 0 || out_layout > 1) return MEEP2B_ERR_SHAPE;
  if (n % 8 || ldg % 8) return MEEP2B_ERR_ALIGN;
  if (!aligned16(g) || !aligned16(low) || !aligned16(out)) return MEEP2B_ERR_ALIGN;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  constexpr int C = 128;  // measured: the 64-column form (twice the CTAs, half the work each) is not faster
  dim3 grid(static_cast<unsigned>((n + C - 1) / C), static_cast<unsigned>(experts));
  reduce::grouped_reduce_kernel<C><<<grid, 2 * C, 0, s>>>(
      static_cast<const __nv_bfloat16*>(g), n, ldg, static_cast<const __nv_bfloat16*>(low), offsets, scaling,
      static_cast<__nv_bfloat16*>(out), g_rows, row_scale, out_layout);
  return launch_status();
}

extern "C" int meep2b_grouped_reduce(const void* g, int64_t rows, int64_t n, int64_t ldg, const void* low,
                                     const int32_t* offsets, int32_t experts, float scaling, void* out,
                                     int32_t out_layout, void* stream) {
  return grouped_reduce_launch(g, nullptr, nullptr, rows, n, ldg, low, offsets, experts, scaling, out, out_layout,
                               stream);
}

extern "C" int meep2b_grouped_reduce_rows(const void* g, const int32_t* g_rows, const float* row_scale,
                                          int64_t rows, int64_t n, int64_t ldg, const void* low,
                                          const int32_t* offsets, int32_t experts, float scaling, void* out,
                                          int32_t out_layout, void* stream) {
  if (g_rows == nullptr) return MEEP2B_ERR_SHAPE;
  return grouped_reduce_launch(g, g_rows, row_scale, rows, n, ldg, low, offsets, experts, scaling, out, out_layout,
                               stream);
}

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

// ---------------------------------------------------------------------------------------------------------------
// Full-row form, for rows read through g_rows (the routed rows of a token-major tensor): a CTA takes a chunk of up
// to FR_CHUNK rows of one expert (the chunk map is the tile map with tiles of FR_CHUNK rows) and all n columns, so
// that each gathered row arrives whole (one bulk copy of n * 2 bytes) instead of as n / 128 pieces of 256 bytes
// fetched by as many CTAs. Warp 8 produces: the chunk's row indices and weights are read into shared memory once,
// then each stage of FR_ROWS rows (one k16 step of the MMAs) goes out as one bulk copy per row (a lane each) plus
// one for the rank panel's rows, on a ring of FR_STAGES stages with full / empty barriers. Warps 0-7 consume: warp
// w owns columns [w * n / 8, (w + 1) * n / 8) (MT m-tiles of 16) and applies the row weights to the panel in
// registers (bf16(w * low), the other form's rounding; rows past the chunk's end weigh nothing). Each chunk writes
// its float32 partial sums (n x 16, row-major) to `partial`; reduce_partials_kernel then adds an expert's chunks in
// order (deterministic) and rounds.
constexpr int FR_ROWS = 16;
constexpr int FR_STAGES = 3;
constexpr int FR_CHUNK = 512;
constexpr int FR_CONSUMERS = 8;  // warps

__host__ __device__ constexpr int fr_gpitch(int n) { return n + 8; }  // bf16 per smem row of g (+16 bytes)
__host__ __device__ constexpr int fr_stage_bytes(int n) { return FR_ROWS * fr_gpitch(n) * 2 + FR_ROWS * 32; }
// stages, then the chunk's row indices and weights (FR_CHUNK each), then 2 x FR_STAGES barriers
__host__ __device__ constexpr int fr_smem_bytes(int n) {
  return FR_STAGES * fr_stage_bytes(n) + FR_CHUNK * 8 + 2 * FR_STAGES * 8;
}

// a bf16 pair times (w0, w1), rounded to bf16; a row past the chunk's end (ok false) gives zero, whatever it holds
__device__ __forceinline__ uint32_t weigh_pair(uint32_t v, float w0, float w1, bool ok0, bool ok1) {
  const float a = ok0 ? __bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>(v & 0xFFFFu))) * w0 : 0.f;
  const float b = ok1 ? __bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>(v >> 16))) * w1 : 0.f;
  return pack_bf16x2(a, b);
}

template <int MT>
__global__ void __launch_bounds__(32 * (FR_CONSUMERS + 1), 1)
    reduce_rows_partial_kernel(const __nv_bfloat16* __restrict__ g, int64_t ldg, const int32_t* __restrict__ g_rows,
                               const float* __restrict__ row_scale, const __nv_bfloat16* __restrict__ low,
                               const int32_t* __restrict__ offsets, const int32_t* __restrict__ chunk_expert,
                               const int32_t* __restrict__ chunk_row, const int32_t* __restrict__ chunks,
                               float* __restrict__ partial) {
  constexpr int N = MT * 16 * FR_CONSUMERS;
  constexpr int GP = fr_gpitch(N);
  constexpr int SB = fr_stage_bytes(N);
  extern __shared__ __align__(128) uint8_t fr_smem[];
  const int c = blockIdx.x;
  if (c >= *chunks) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = chunk_expert[c];
  const int64_t r0 = chunk_row[c];
  const int count = static_cast<int>(min(static_cast<int64_t>(FR_CHUNK), static_cast<int64_t>(offsets[e]) - r0));
  const int steps = (count + FR_ROWS - 1) / FR_ROWS;
  const uint32_t sbase = smem_u32(fr_smem);
  int32_t* idx_s = reinterpret_cast<int32_t*>(fr_smem + FR_STAGES * SB);
  float* w_s = reinterpret_cast<float*>(fr_smem + FR_STAGES * SB + FR_CHUNK * 4);
  const uint32_t full0 = sbase + FR_STAGES * SB + FR_CHUNK * 8;
  const uint32_t empty0 = full0 + 8u * FR_STAGES;
  // every stage zero first, so that rows past the chunk's end hold finite values (zeros or earlier rows of the
  // chunk); the chunk's row indices and weights (1 when unweighted) into shared memory
  for (int i = threadIdx.x; i < FR_STAGES * SB / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(fr_smem)[i] = make_uint4(0, 0, 0, 0);
  for (int i = threadIdx.x; i < count; i += blockDim.x) {
    idx_s[i] = g_rows != nullptr ? g_rows[r0 + i] : static_cast<int32_t>(r0 + i);
    w_s[i] = row_scale != nullptr ? row_scale[r0 + i] : 1.f;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < FR_STAGES; ++s) {
      mbar_init(full0 + 8u * s, 1);
      mbar_init(empty0 + 8u * s, FR_CONSUMERS);
    }
    fence_barrier_init();
  }
  fence_proxy_async_smem();
  __syncthreads();
  auto rows_of = [&](int step) { return min(FR_ROWS, count - step * FR_ROWS); };

  bool failed = false;
  int issued = 0;  // producer: steps whose copies went out
  if (warp == FR_CONSUMERS) {
    for (int step = 0; step < steps; ++step) {
      const int s = step % FR_STAGES;
      if (step >= FR_STAGES && !mbar_wait(empty0 + 8u * s, static_cast<uint32_t>((step / FR_STAGES - 1) & 1))) {
        failed = true;
        break;
      }
      const int rows = rows_of(step);
      const uint32_t bar = full0 + 8u * s;
      if (lane == 0) mbar_arrive_expect_tx(bar, static_cast<uint32_t>(rows) * (N * 2 + 32));
      __syncwarp();
      if (lane < rows)
        bulk_load(sbase + s * SB + lane * GP * 2, g + static_cast<int64_t>(idx_s[step * FR_ROWS + lane]) * ldg,
                  N * 2, bar);
      if (lane == 0)
        bulk_load(sbase + s * SB + FR_ROWS * GP * 2, low + (r0 + step * FR_ROWS) * 16,
                  static_cast<uint32_t>(rows) * 32, bar);
      issued = step + 1;
    }
  }

  float acc[MT][2][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int h = 0; h < 2; ++h) acc[m][h][0] = acc[m][h][1] = acc[m][h][2] = acc[m][h][3] = 0.f;
  if (warp < FR_CONSUMERS) {
    const int q = lane & 3;
    for (int step = 0; step < steps; ++step) {
      const int s = step % FR_STAGES;
      if (!__all_sync(0xffffffffu, mbar_wait(full0 + 8u * s, static_cast<uint32_t>((step / FR_STAGES) & 1)))) {
        failed = true;
        break;
      }
      const int rows = rows_of(step);
      const __nv_bfloat16* ls = reinterpret_cast<const __nv_bfloat16*>(fr_smem + s * SB + FR_ROWS * GP * 2);
      // B (16 rows x 16 ranks) = the panel: blocks (rows 0-7 | 8-15) x (ranks 0-7 | 8-15), transposed; the lane
      // holds rows 2q, 2q + 1 (b[0], b[2]) and 2q + 8, 2q + 9 (b[1], b[3]) of rank lane / 4 (+ 8)
      uint32_t b[4];
      {
        const int mtx = lane >> 3, rr = lane & 7;
        ldmatrix_x4_trans(b, ls + ((mtx & 1) * 8 + rr) * 16 + (mtx >> 1) * 8);
      }
      {
        const float* ws = w_s + step * FR_ROWS;
        const int k0 = 2 * q, k1 = 2 * q + 8;
        const float w0 = ws[k0], w1 = ws[k0 + 1], w2 = ws[k1], w3 = ws[k1 + 1];
        b[0] = weigh_pair(b[0], w0, w1, k0 < rows, k0 + 1 < rows);
        b[2] = weigh_pair(b[2], w0, w1, k0 < rows, k0 + 1 < rows);
        b[1] = weigh_pair(b[1], w2, w3, k1 < rows, k1 + 1 < rows);
        b[3] = weigh_pair(b[3], w2, w3, k1 < rows, k1 + 1 < rows);
      }
      const __nv_bfloat16* gs = reinterpret_cast<const __nv_bfloat16*>(fr_smem + s * SB);
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        // A (16 columns x 16 rows) = g^T
        uint32_t a[4];
        const int mtx = lane >> 3, rr = lane & 7;
        const int row = (mtx >> 1) * 8 + rr;
        const int col = (warp * MT + m) * 16 + (mtx & 1) * 8;
        ldmatrix_x4_trans(a, gs + row * GP + col);
        mma16816(acc[m][0], a, b[0], b[1]);
        mma16816(acc[m][1], a, b[2], b[3]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty0 + 8u * s);  // stage s is free again
    }
  }
  if (__syncthreads_or(failed)) {
    // a wait gave up (the error is recorded): the producer waits (bounded) for the copies of its last stages,
    // which may still be in flight, before the CTA's shared memory goes away; no partial sums are written
    if (warp == FR_CONSUMERS && lane == 0)
      for (int st = max(0, issued - FR_STAGES); st < issued; ++st)
        mbar_wait_drain(full0 + 8u * (st % FR_STAGES), static_cast<uint32_t>((st / FR_STAGES) & 1));
    __syncthreads();
    return;
  }
  if (warp >= FR_CONSUMERS) return;
  // partial[c][col][rank]: C fragment c0,c1 -> (column = lane / 4, ranks 2 (lane % 4) + {0, 1}); c2,c3 -> column + 8
  float* out = partial + static_cast<int64_t>(c) * N * 16;
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    const int col = (warp * MT + m) * 16 + (lane >> 2);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int rk = h * 8 + 2 * (lane & 3);
      *reinterpret_cast<float2*>(out + col * 16 + rk) = make_float2(acc[m][h][0], acc[m][h][1]);
      *reinterpret_cast<float2*>(out + (col + 8) * 16 + rk) = make_float2(acc[m][h][2], acc[m][h][3]);
    }
  }
}

// out[e] = bf16(scaling * sum over expert e's chunks, in order, of partial[chunk]); a thread per column and four
// ranks (one float4 per chunk, the loads of up to four chunks in flight). The expert's chunks are consecutive in
// the chunk map.
__global__ void __launch_bounds__(128) reduce_partials_kernel(const float* __restrict__ partial, int n,
                                                              const int32_t* __restrict__ offsets, int chunk_rows,
                                                              float scaling, __nv_bfloat16* __restrict__ out,
                                                              int out_layout) {
  const int e = blockIdx.y;
  __shared__ int first_s;
  if (threadIdx.x < 32) {  // the chunks of the experts before e, summed by one warp
    int sum = 0;
    for (int i = threadIdx.x; i < e; i += 32) {
      const int rows = offsets[i] - (i > 0 ? offsets[i - 1] : 0);
      sum += (rows + chunk_rows - 1) / chunk_rows;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (threadIdx.x == 0) first_s = sum;
  }
  __syncthreads();
  const int first = first_s;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;  // column t / 4, ranks 4 (t % 4) + [0, 4)
  if (t >= n * 4) return;
  const int col = t >> 2, r0 = (t & 3) * 4;
  const int rows_e = offsets[e] - (e > 0 ? offsets[e - 1] : 0);
  const int count = (rows_e + chunk_rows - 1) / chunk_rows;
  const float4* src = reinterpret_cast<const float4*>(partial) + static_cast<int64_t>(first) * n * 4 + t;
  const int64_t stride = static_cast<int64_t>(n) * 4;  // float4 per chunk
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k = 0; k < count; k += 4) {
    float4 p[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) p[j] = k + j < count ? src[(k + j) * stride] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (k + j < count) {
        v.x = __fadd_rn(v.x, p[j].x);
        v.y = __fadd_rn(v.y, p[j].y);
        v.z = __fadd_rn(v.z, p[j].z);
        v.w = __fadd_rn(v.w, p[j].w);
      }
    }
  }
  __nv_bfloat16* o = out + static_cast<int64_t>(e) * n * 16;
  if (out_layout == 0) {
    *reinterpret_cast<uint2*>(o + static_cast<int64_t>(col) * 16 + r0) =
        make_uint2(pack_bf16x2(v.x * scaling, v.y * scaling), pack_bf16x2(v.z * scaling, v.w * scaling));
  } else {
    o[static_cast<int64_t>(r0) * n + col] = __float2bfloat16_rn(v.x * scaling);
    o[static_cast<int64_t>(r0 + 1) * n + col] = __float2bfloat16_rn(v.y * scaling);
    o[static_cast<int64_t>(r0 + 2) * n + col] = __float2bfloat16_rn(v.z * scaling);
    o[static_cast<int64_t>(r0 + 3) * n + col] = __float2bfloat16_rn(v.w * scaling);
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

extern "C" int meep2b_grouped_reduce_rows_full(const void* g, const int32_t* g_rows, const float* row_scale,
                                               int64_t rows, int64_t n, int64_t ldg, const void* low,
                                               const int32_t* offsets, int32_t experts, float scaling, void* out,
                                               int32_t out_layout, const int32_t* chunk_expert,
                                               const int32_t* chunk_row, const int32_t* chunks, int64_t max_chunks,
                                               float* partial, size_t partial_bytes, void* stream) {
  using namespace meep2b;
  using namespace meep2b::reduce;
  if (rows < 0 || experts < 1 || ldg < n || out_layout < 0 || out_layout > 1 || max_chunks < 0)
    return MEEP2B_ERR_SHAPE;
  if (rows > INT32_MAX) return MEEP2B_ERR_SHAPE;
  if (n != 768 && n != 1536 && n != 2048) return MEEP2B_ERR_UNSUPPORTED;
  if (ldg % 8) return MEEP2B_ERR_ALIGN;
  if (!aligned16(g) || !aligned16(low) || !aligned16(out) || !aligned16(partial)) return MEEP2B_ERR_ALIGN;
  if (partial_bytes < static_cast<size_t>(max_chunks) * static_cast<size_t>(n) * 16 * sizeof(float))
    return MEEP2B_ERR_SHAPE;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  if (rows == 0) {
    cudaMemsetAsync(out, 0, static_cast<size_t>(experts) * n * 16 * 2, s);
    return launch_status();
  }
  const int smem = fr_smem_bytes(static_cast<int>(n));
  auto run = [&](auto kern) -> int {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
      cudaGetLastError();
      return MEEP2B_ERR_LAUNCH;
    }
    kern<<<static_cast<unsigned>(max_chunks > 0 ? max_chunks : 1), 32 * (FR_CONSUMERS + 1), smem, s>>>(
        static_cast<const __nv_bfloat16*>(g), ldg, g_rows, row_scale, static_cast<const __nv_bfloat16*>(low), offsets,
        chunk_expert, chunk_row, chunks, partial);
    return launch_status();
  };
  int st;
  if (n == 768) st = run(reduce_rows_partial_kernel<6>);
  else if (n == 1536) st = run(reduce_rows_partial_kernel<12>);
  else st = run(reduce_rows_partial_kernel<16>);
  if (st != MEEP2B_OK) return st;
  dim3 grid(static_cast<unsigned>((n * 4 + 127) / 128), static_cast<unsigned>(experts));
  reduce_partials_kernel<<<grid, 128, 0, s>>>(partial, static_cast<int>(n), offsets, FR_CHUNK, scaling,
                                               static_cast<__nv_bfloat16*>(out), out_layout);
  return launch_status();
}

extern "C" int meep2b_reduce_chunk_rows(void) { return meep2b::reduce::FR_CHUNK; }

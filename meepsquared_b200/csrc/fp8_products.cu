// FP8 tensor-core products of an e4m3 expert stack: the reference's X_FP8 path (_grouped.py:141-146,194-197),
// which MEEPSQUARED_FP8_PRODUCTS=1 or products_fp8=True selects (_grouped.py:70-80,316-320).
//
// The reference quantises each x tile per row to e4m3 by the row's largest magnitude over the tile's K columns,
// multiplies the codes with the stack's codes on the FP8 tensor cores, and undoes the row scale on the tile's
// partial product before adding it to the float32 accumulator; the per-expert scale multiplies the sum.  Here:
//
//  * quantize_rows_kernel: x (rows, k) bf16 -> codes (rows, k) e4m3 and scales (k/128 blocks, rows) float32,
//    scale = max(amax over the row's 128 columns of the block, 1e-12) / 448, code = e4m3(x / scale) (round to
//    nearest even); eight lanes per (row, block), 2 bytes read and 1 written per element.
//  * grouped_gemm_f8_kernel: persistent, one CTA per SM, one unit = 128 rows of one expert x 256 columns.
//    Warp 0 loads the x codes and the stack's codes with TMA (128 x 128 and 256 x 128 bytes per k-block,
//    128-byte swizzle); warp 1 issues tcgen05.mma kind::f8f6f4 (e4m3 x e4m3, float32 accumulation), four MMAs of depth 32
//    per 128-column k-block, each k-block into its own tensor-memory buffer (2 buffers of 256 columns); warps
//    2-9 promote: each thread owns one row and 128 columns of the unit in registers and adds every k-block's
//    partial sum times the row's scale of that block (times the stack's block scale, for block-scaled stacks).
//    The adapters' up product (the bf16 panel x A^T, computed beforehand, times U) is one more bf16 MMA of depth
//    16 into a buffer, added with the factor s. The epilogue applies the per-expert scale, the bias, rounds to
//    bf16 and stores the row's 128 columns.
// Every wait is bounded (common.cuh): a role that gives up records MEEP2B_ERR_TIMEOUT and the kernel returns.
#include <cuda_fp8.h>

namespace meep2b {
namespace f8 {

constexpr int BM = 128, BN = 256, BK = 128;  // BK is also the activations' quantisation block
constexpr int STAGES = 4;
constexpr int NBUF = 2;       // partial-sum buffers in tensor memory, 256 columns each
constexpr int THREADS = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 promotion and epilogue (no idle warps: the
                              // promotion's 128 float32 accumulators a thread need the registers)
constexpr int PROMO_WARP0 = 2;
constexpr int PROMO_WARPS = 8;
constexpr int COLS = BN / 2;  // columns of a unit one promotion thread owns
constexpr uint32_t A_BYTES = BM * BK;
constexpr uint32_t B_BYTES = BN * BK;
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
constexpr uint32_t LOW_BYTES = BM * 16 * 2;
constexpr uint32_t U_BYTES = BN * 16 * 2;
constexpr uint32_t OFF_LOW = STAGES * STAGE_BYTES;
constexpr uint32_t OFF_U = OFF_LOW + LOW_BYTES;
constexpr uint32_t OFF_BAR = OFF_U + U_BYTES;
constexpr uint32_t N_BARS = 2 * STAGES + 2 * NBUF + 3;
constexpr uint32_t OFF_TMEM = OFF_BAR + 8 * N_BARS;
constexpr uint32_t SMEM_BYTES = OFF_TMEM + 16 + 1024;  // + the slack of aligning the base to 1024 bytes
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory of one CTA");
constexpr uint32_t TMEM_COLS = NBUF * BN;
static_assert(TMEM_COLS <= 512, "tensor memory columns");

struct Params {
  int rows, K, N, kblocks, nblocks;
  int64_t ldo;
  const float* xscale;  // (kblocks, ld_xscale): the scale of row r over k-block kb at xscale[kb * ld_xscale + r]
  int64_t ld_xscale;
  const float* scale;   // (experts,) or null
  const float* wblock;  // block scales of the stack or null: wblock[e * se + (kb / div_k) * sk + (c / div_n) * sn],
                        // c = column / 128
  int64_t wb_se, wb_sk, wb_sn;
  int wb_div_k, wb_div_n;
  const __nv_bfloat16* bias;  // (experts, N) or null
  float scaling;
  const int32_t* offsets;
  const int32_t* tile_expert;
  const int32_t* tile_row;
  const int32_t* tiles;
  __nv_bfloat16* out;
};

// Instruction descriptor of kind::f8f6f4 with e4m3 A and B (format code 0), a float32 accumulator, M x N.
__host__ __device__ constexpr uint32_t idesc_e4m3(int m, int n, bool b_mn) {
  return (1u << 4) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_e4m3(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// 32 lanes x 64 columns of 32-bit in one load; one wait.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, "
      "%36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, "
      "%57, %58, %59, %60, %61, %62, %63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr));
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// The e4m3 codes (round to nearest even, saturating) of x0 / s and x1 / s, the quotients rounded to float32 as a
// division rounds them, without a division for almost every element: q = |x| * rcp (rcp = 1 / s correctly rounded)
// is within 2.5 ulp of the rounded quotient, and rounding to e4m3 is monotonic, so when the codes of q - 6 ulp and
// q + 6 ulp agree the quotient has that code too. Only near a rounding midpoint of e4m3 (6 ulp in 2^20 of each
// code's interval) is the quotient computed by division. The sign is the sign of x, as a cast keeps it.
__device__ __forceinline__ uint32_t e4m3_pair(float a, float b) {
  return static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3));
}

__device__ __forceinline__ uint32_t e4m3_quotients(float x0, float x1, float s, float rcp) {
  const float a0 = fabsf(x0), a1 = fabsf(x1);
  const uint32_t b0 = __float_as_uint(a0 * rcp), b1 = __float_as_uint(a1 * rcp);
  const uint32_t lo = e4m3_pair(__uint_as_float(b0 > 6u ? b0 - 6u : 0u), __uint_as_float(b1 > 6u ? b1 - 6u : 0u));
  const uint32_t hi = e4m3_pair(__uint_as_float(b0 + 6u), __uint_as_float(b1 + 6u));
  const uint32_t mag = lo == hi ? lo : e4m3_pair(a0 / s, a1 / s);
  return mag | ((__float_as_uint(x0) >> 24) & 0x80u) | ((__float_as_uint(x1) >> 16) & 0x8000u);
}

// Eight lanes per (row, 128-column block), lane i of the eight holding columns 16i..16i+15 of the block (two
// 16-byte loads); each group issues the loads of two blocks before it uses any, so 64 bytes a lane are in flight.
// A block's two divisions (its scale and the scale's reciprocal) and its max reduction are shared by 16 elements a
// lane.
constexpr int Q_UNROLL = 2;
constexpr int Q_LANES = 8;

__global__ void __launch_bounds__(256) quantize_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows, int k,
                                                            int64_t ldx, uint8_t* __restrict__ codes,
                                                            float* __restrict__ scales, int64_t ld_scales) {
  const int kblocks = (k + BK - 1) / BK;
  const int64_t items = rows * kblocks;
  const bool small = items + static_cast<int64_t>(Q_UNROLL) * gridDim.x * blockDim.x < (int64_t(1) << 32);
  const int sub = threadIdx.x & (Q_LANES - 1);
  const int64_t group = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / Q_LANES;
  const int64_t groups = (static_cast<int64_t>(gridDim.x) * blockDim.x) / Q_LANES;
  constexpr int PER_WARP = 32 / Q_LANES;
  // the loop bound is the warp's first group's (groups is a multiple of PER_WARP), so all groups of a warp take
  // the same trips and every full-mask shuffle has all 32 lanes; items past the end are masked by `valid`
  for (int64_t warp_base = group & ~int64_t(PER_WARP - 1); warp_base < items; warp_base += Q_UNROLL * groups) {
    const int64_t base = warp_base + (group & (PER_WARP - 1));
    uint4 raw[Q_UNROLL][2];
    int64_t row[Q_UNROLL];
    int kb[Q_UNROLL];
    bool in[Q_UNROLL];
#pragma unroll
    for (int u = 0; u < Q_UNROLL; ++u) {
      const int64_t item = base + u * groups;
      const bool valid = item < items;
      // a 32-bit division where the item count allows (a 64-bit one is a long emulated sequence)
      row[u] = !valid ? 0 : (small ? static_cast<int64_t>(static_cast<uint32_t>(item) / static_cast<uint32_t>(kblocks))
                                   : item / kblocks);
      kb[u] = valid ? static_cast<int>(item - row[u] * kblocks) : 0;
      const int col = kb[u] * BK + sub * 16;
      in[u] = valid && col < k;  // k is a multiple of 16: a lane's sixteen columns are all in range or all out
      const uint4* src = reinterpret_cast<const uint4*>(x + row[u] * ldx + col);
      raw[u][0] = in[u] ? __ldg(src) : make_uint4(0, 0, 0, 0);
      raw[u][1] = in[u] ? __ldg(src + 1) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < Q_UNROLL; ++u) {
      const uint32_t w[8] = {raw[u][0].x, raw[u][0].y, raw[u][0].z, raw[u][0].w,
                             raw[u][1].x, raw[u][1].y, raw[u][1].z, raw[u][1].w};
      float v[16];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[2 * i] = bf16_lo(w[i]), v[2 * i + 1] = bf16_hi(w[i]);
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
      for (int o = Q_LANES / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float s = fmaxf(amax, 1e-12f) / 448.0f;
      if (in[u]) {
        const float rcp = 1.0f / s;
        uint32_t q[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = e4m3_quotients(v[2 * i], v[2 * i + 1], s, rcp);
        *reinterpret_cast<uint4*>(codes + row[u] * k + kb[u] * BK + sub * 16) =
            make_uint4(q[0] | (q[1] << 16), q[2] | (q[3] << 16), q[4] | (q[5] << 16), q[6] | (q[7] << 16));
      }
      if (sub == 0 && base + u * groups < items) scales[static_cast<int64_t>(kb[u]) * ld_scales + row[u]] = s;
    }
  }
}

template <bool B_MN, bool LORA>
__global__ void __launch_bounds__(THREADS, 1)
    grouped_gemm_f8_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                           const __grid_constant__ CUtensorMap tm_low, const __grid_constant__ CUtensorMap tm_u,
                           const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const uint32_t bar0 = sbase + OFF_BAR;
  auto bar_full = [&](int s) { return bar0 + 8u * s; };
  auto bar_empty = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto bar_pfull = [&](int b) { return bar0 + 8u * (2 * STAGES + b); };
  auto bar_pempty = [&](int b) { return bar0 + 8u * (2 * STAGES + NBUF + b); };
  const uint32_t bar_lfull = bar0 + 8u * (2 * STAGES + 2 * NBUF);
  const uint32_t bar_lempty = bar0 + 8u * (2 * STAGES + 2 * NBUF + 1);
  const uint32_t bar_drain = bar0 + 8u * (2 * STAGES + 2 * NBUF + 2);  // only on the way out of a failed run
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_TMEM);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full(s), 1);
      mbar_init(bar_empty(s), 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(bar_pfull(b), 1);
      mbar_init(bar_pempty(b), PROMO_WARPS);
    }
    mbar_init(bar_lfull, 1);
    mbar_init(bar_lempty, 1);
    mbar_init(bar_drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total = (*p.tiles) * p.nblocks;

  if (warp == 0) {
    // ------------------------------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_w);
      if (LORA) {
        tma_prefetch_desc(&tm_low);
        tma_prefetch_desc(&tm_u);
      }
      int stage = 0;
      uint32_t phase = 0;
      uint32_t last_parity[STAGES];
      bool issued[STAGES];
      for (int s = 0; s < STAGES; ++s) issued[s] = false, last_parity[s] = 0;
      bool l_issued = false;
      uint32_t l_parity = 0;
      bool ok = true;
      int it = 0;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ++it) {
        const int t = u / p.nblocks, nb = u - t * p.nblocks;
        const int e = p.tile_expert[t], row0 = p.tile_row[t];
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait(bar_empty(stage), phase ^ 1)) { ok = false; break; }
          const uint32_t fb = bar_full(stage);
          const uint32_t a_dst = sbase + stage * STAGE_BYTES;
          const uint32_t b_dst = a_dst + A_BYTES;
          mbar_arrive_expect_tx(fb, STAGE_BYTES);
          tma_load_2d(a_dst, &tm_x, fb, kb * BK, row0);
          if (B_MN) {  // two boxes of 128 columns (the 128-byte swizzle spans 128 codes)
            tma_load_3d(b_dst, &tm_w, fb, nb * BN, kb * BK, e);
            tma_load_3d(b_dst + BK * 128, &tm_w, fb, nb * BN + 128, kb * BK, e);
          } else {
            tma_load_3d(b_dst, &tm_w, fb, kb * BK, nb * BN, e);
          }
          issued[stage] = true;
          last_parity[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if (LORA) {
          if (!mbar_wait(bar_lempty, (it & 1) ^ 1)) { ok = false; break; }
          mbar_arrive_expect_tx(bar_lfull, LOW_BYTES + U_BYTES);
          tma_load_2d(sbase + OFF_LOW, &tm_low, bar_lfull, 0, row0);
          tma_load_3d(sbase + OFF_U, &tm_u, bar_lfull, 0, nb * BN, e);
          l_issued = true;
          l_parity = it & 1;
        }
      }
      if (!ok) {
        // a partner is gone: let this thread's copies in flight land before the CTA's shared memory goes away
        for (int s = 0; s < STAGES; ++s)
          if (issued[s]) mbar_wait_drain(bar_full(s), last_parity[s]);
        if (l_issued) mbar_wait_drain(bar_lfull, l_parity);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_e4m3(BM, BN, B_MN);
      constexpr uint32_t IDESC_UP = idesc_bf16(BM, BN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t g = 0;  // partial sums issued so far: buffer g % NBUF, its use number g / NBUF
      bool ok = true;
      int it = 0;
      auto take_buffer = [&]() -> uint32_t {
        const uint32_t b = g % NBUF;
        if (!mbar_wait(bar_pempty(b), ((g / NBUF) & 1) ^ 1)) return 0xFFFFFFFFu;
        tc_fence_after();
        return b;
      };
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ++it) {
        for (int kb = 0; kb < p.kblocks; ++kb) {
          const uint32_t b = take_buffer();
          if (b == 0xFFFFFFFFu || !mbar_wait(bar_full(stage), phase)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d = tmem_base + b * BN;
          const uint32_t a_addr = sbase + stage * STAGE_BYTES;
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk) {
            const uint64_t adesc = smem_desc(a_addr + kk * 32, 16, 1024, 2);
            const uint64_t bdesc =
                B_MN ? smem_desc(b_addr + kk * 4096, BK * 128, 1024, 2) : smem_desc(b_addr + kk * 32, 16, 1024, 2);
            mma_e4m3(d, adesc, bdesc, IDESC, kk != 0);
          }
          mma_commit(bar_empty(stage));
          mma_commit(bar_pfull(b));
          ++g;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if (LORA) {
          const uint32_t b = take_buffer();
          if (b == 0xFFFFFFFFu || !mbar_wait(bar_lfull, it & 1)) { ok = false; break; }
          tc_fence_after();
          mma_bf16(tmem_base + b * BN, smem_desc(sbase + OFF_LOW, 16, 256, 6), smem_desc(sbase + OFF_U, 16, 256, 6),
                   IDESC_UP, 0);
          mma_commit(bar_lempty);
          mma_commit(bar_pfull(b));
          ++g;
        }
      }
      if (!ok) {
        // let the MMAs already issued finish before tensor memory is released
        mma_commit(bar_drain);
        mbar_wait_drain(bar_drain, 0);
      }
    }
  } else if (warp >= PROMO_WARP0) {
    // ------------------------------------------------------------------------------------------ promotion
    const int q = warp & 3;                          // TMEM lane quarter this warp may read
    const int half = (warp - PROMO_WARP0) >> 2;      // which 128 of the unit's 256 columns
    const int r = q * 32 + lane;                     // the thread's row within the unit
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    uint32_t g = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
      const int t = u / p.nblocks, nb = u - t * p.nblocks;
      const int e = p.tile_expert[t], row0 = p.tile_row[t];
      const int row = row0 + r;
      const int row_end = min(p.offsets[e], p.rows);
      const int row_c = min(row, p.rows - 1);
      float acc[COLS];
#pragma unroll
      for (int j = 0; j < COLS; ++j) acc[j] = 0.f;
      const int cblock = nb * (BN / 128) + half;  // the 128-column block of the thread's columns
      auto factor_of = [&](int kb) -> float {
        if (LORA && kb == p.kblocks) return p.scaling;  // the adapters' up product, after the base's k-blocks
        float f = __ldg(p.xscale + static_cast<int64_t>(kb) * p.ld_xscale + row_c);
        if (p.wblock != nullptr)
          f *= __ldg(p.wblock + e * p.wb_se + (kb / p.wb_div_k) * p.wb_sk + (cblock / p.wb_div_n) * p.wb_sn);
        return f;
      };
      const int steps = p.kblocks + (LORA ? 1 : 0);
      const float se = p.scale != nullptr ? __ldg(p.scale + e) : 1.f;
      float f_next = factor_of(0);  // each k-block's scale is loaded one k-block ahead, off the wait's path
      for (int kb = 0; kb < steps; ++kb) {
        const float f = f_next;
        if (kb + 1 < steps) f_next = factor_of(kb + 1);
        if (kb == p.kblocks) {  // the base sum is complete: the per-expert scale, then the adapters' product
#pragma unroll
          for (int j = 0; j < COLS; ++j) acc[j] *= se;
        }
        const uint32_t b = g % NBUF;
        if (!mbar_wait(bar_pfull(b), (g / NBUF) & 1)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < COLS; c += 16) {
          float v[16];
          tmem_ld16(tmem_base + lane_addr + b * BN + half * COLS + c, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[c + j] = fmaf(v[j], f, acc[c + j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_pempty(b));
        ++g;
      }
      if (!ok) break;
      if (!LORA) {
#pragma unroll
        for (int j = 0; j < COLS; ++j) acc[j] *= se;
      }
      const int col0 = nb * BN + half * COLS;
      if (p.bias != nullptr) {
        const __nv_bfloat16* bias = p.bias + static_cast<int64_t>(e) * p.N + col0;
#pragma unroll
        for (int j = 0; j < COLS; j += 8) {
          if (col0 + j < p.N) {
            const uint4 w = __ldg(reinterpret_cast<const uint4*>(bias + j));
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              acc[j + 2 * i] += bf16_lo(ws[i]);
              acc[j + 2 * i + 1] += bf16_hi(ws[i]);
            }
          }
        }
      }
      if (row < row_end) {
        __nv_bfloat16* dst = p.out + static_cast<int64_t>(row) * p.ldo + col0;
#pragma unroll
        for (int j = 0; j < COLS; j += 8) {
          if (col0 + j < p.N) {
            uint4 w;
            w.x = pack_bf16x2(acc[j], acc[j + 1]);
            w.y = pack_bf16x2(acc[j + 2], acc[j + 3]);
            w.z = pack_bf16x2(acc[j + 4], acc[j + 5]);
            w.w = pack_bf16x2(acc[j + 6], acc[j + 7]);
            *reinterpret_cast<uint4*>(dst + j) = w;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <bool B_MN, bool LORA>
static int launch(const CUtensorMap& tx, const CUtensorMap& tw, const CUtensorMap& tl, const CUtensorMap& tu,
                  const Params& prm, int grid, cudaStream_t s) {
  auto kern = grouped_gemm_f8_kernel<B_MN, LORA>;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess) {
      cudaGetLastError();
      return MEEP2B_ERR_LAUNCH;
    }
    configured = true;
  }
  kern<<<grid, THREADS, SMEM_BYTES, s>>>(tx, tw, tl, tu, prm);
  return launch_status();
}

}  // namespace f8
}  // namespace meep2b

extern "C" int meep2b_fp8_rows_quantize(const void* x, int64_t rows, int64_t k, int64_t ldx, uint8_t* codes,
                                        float* scales, int64_t ld_scales, void* stream) {
  using namespace meep2b;
  if (rows < 0 || k < 1 || ldx < k || ld_scales < rows || k > INT32_MAX) return MEEP2B_ERR_SHAPE;
  if (k % 16 || ldx % 8) return MEEP2B_ERR_ALIGN;
  if (!aligned16(x) || !aligned16(codes) || (reinterpret_cast<uintptr_t>(scales) & 3u)) return MEEP2B_ERR_ALIGN;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  if (rows == 0) return MEEP2B_OK;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t items = rows * ((k + f8::BK - 1) / f8::BK);
  const int64_t per_block = (256 / f8::Q_LANES) * f8::Q_UNROLL;  // items a block takes per trip
  const int64_t blocks = (items + per_block - 1) / per_block;
  const int grid = static_cast<int>(blocks < int64_t(sms) * 8 ? blocks : int64_t(sms) * 8);
  f8::quantize_rows_kernel<<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), rows, static_cast<int>(k), ldx,
                                                codes, scales, ld_scales);
  return launch_status();
}

extern "C" int meep2b_grouped_product_f8(const meep2b_product_f8* a, void* stream) {
  using namespace meep2b;
  if (a == nullptr) return MEEP2B_ERR_SHAPE;
  if (a->rows < 0 || a->k < 1 || a->n < 1 || a->experts < 1) return MEEP2B_ERR_SHAPE;
  if (a->rows > INT32_MAX || a->k > INT32_MAX || a->n > INT32_MAX) return MEEP2B_ERR_SHAPE;
  if (a->k % 16 || a->n % 16 || a->ldo % 8 || a->ldo < a->n || a->ld_xscale < a->rows) return MEEP2B_ERR_ALIGN;
  const bool lora = a->low != nullptr;
  if (lora && a->up == nullptr) return MEEP2B_ERR_SHAPE;
  if (a->wblock != nullptr && (a->wb_div_k < 1 || a->wb_div_n < 1)) return MEEP2B_ERR_SHAPE;
  if (!aligned16(a->x8) || !aligned16(a->weight) || !aligned16(a->out) || (a->bias && !aligned16(a->bias)) ||
      (lora && (!aligned16(a->low) || !aligned16(a->up))))
    return MEEP2B_ERR_ALIGN;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  if (a->rows == 0) return MEEP2B_OK;

  const uint64_t K = a->k, N = a->n, E = a->experts, rows = a->rows;
  CUtensorMap tx, tw, tl, tu;
  {
    const uint64_t dims[2] = {K, rows};
    const uint64_t strides[1] = {K};
    const uint32_t box[2] = {f8::BK, f8::BM};
    MEEP2B_TRY(encode_tiled(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a->x8, dims, strides, box,
                            CU_TENSOR_MAP_SWIZZLE_128B));
  }
  if (!a->b_mn) {
    const uint64_t dims[3] = {K, N, E};
    const uint64_t strides[2] = {K, N * K};
    const uint32_t box[3] = {f8::BK, f8::BN, 1};
    MEEP2B_TRY(encode_tiled(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, a->weight, dims, strides, box,
                            CU_TENSOR_MAP_SWIZZLE_128B));
  } else {
    const uint64_t dims[3] = {N, K, E};
    const uint64_t strides[2] = {N, K * N};
    const uint32_t box[3] = {128, f8::BK, 1};  // two loads of 128 columns per tile
    MEEP2B_TRY(encode_tiled(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, a->weight, dims, strides, box,
                            CU_TENSOR_MAP_SWIZZLE_128B));
  }
  if (lora) {
    const uint64_t ld[2] = {16, rows};
    const uint64_t ls[1] = {32};
    const uint32_t lb[2] = {16, f8::BM};
    MEEP2B_TRY(encode_tiled(&tl, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a->low, ld, ls, lb, CU_TENSOR_MAP_SWIZZLE_32B));
    const uint64_t ud[3] = {16, N, E};
    const uint64_t us[2] = {32, N * 32};
    const uint32_t ub[3] = {16, f8::BN, 1};
    MEEP2B_TRY(encode_tiled(&tu, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a->up, ud, us, ub, CU_TENSOR_MAP_SWIZZLE_32B));
  } else {
    tl = tx;
    tu = tx;
  }

  f8::Params prm;
  prm.rows = static_cast<int>(rows);
  prm.K = static_cast<int>(K);
  prm.N = static_cast<int>(N);
  prm.kblocks = static_cast<int>((K + f8::BK - 1) / f8::BK);
  prm.nblocks = static_cast<int>((N + f8::BN - 1) / f8::BN);
  prm.ldo = a->ldo;
  prm.xscale = a->xscale;
  prm.ld_xscale = a->ld_xscale;
  prm.scale = a->scale;
  prm.wblock = a->wblock;
  prm.wb_se = a->wb_stride_e;
  prm.wb_sk = a->wb_stride_k;
  prm.wb_sn = a->wb_stride_n;
  prm.wb_div_k = a->wblock ? a->wb_div_k : 1;
  prm.wb_div_n = a->wblock ? a->wb_div_n : 1;
  prm.bias = static_cast<const __nv_bfloat16*>(a->bias);
  prm.scaling = a->scaling;
  prm.offsets = a->offsets;
  prm.tile_expert = a->tile_expert;
  prm.tile_row = a->tile_row;
  prm.tiles = a->tiles;
  prm.out = static_cast<__nv_bfloat16*>(a->out);

  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (a->sm_limit > 0 && a->sm_limit < sms) sms = a->sm_limit;
  const int64_t units = a->max_tiles * prm.nblocks;
  const int grid = static_cast<int>(units < sms ? (units > 0 ? units : 1) : sms);
  if (a->b_mn) return lora ? f8::launch<true, true>(tx, tw, tl, tu, prm, grid, s) : f8::launch<true, false>(tx, tw, tl, tu, prm, grid, s);
  return lora ? f8::launch<false, true>(tx, tw, tl, tu, prm, grid, s) : f8::launch<false, false>(tx, tw, tl, tu, prm, grid, s);
}

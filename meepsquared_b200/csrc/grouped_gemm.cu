// The grouped product of the expert layer on sm_100a: a persistent, warp-specialised tcgen05 GEMM.
//
// Replaces _grouped_gemm_kernel and _launch (meepsquared/_grouped.py:121-221, 313-345). Rows are sorted by expert;
// a work unit is (tile of 128 rows of one expert, block of 192 output columns). Per CTA (one per SM, 12 warps):
//   warp 0      TMA producer: x tile (128 x 64), the stack tile (192 x 64) with the rank-16 adapter panel P_e
//               riding along as 16 extra rows (K-major) or a 4th column chunk (MN-major); a ring of 5 (K-major)
//               or 4 (MN-major) stages; after a unit's k-steps, the adapter's up factor U_e for its columns;
//   warp 1      TMEM owner and MMA issuer: per k-step 4 x tcgen05.mma M=128 N=208 K=16 into one of two
//               accumulators (columns 0..191 the product, 192..207 the panel low = x P_e^T); at the end of the
//               unit two more MMAs of depth 16 add (s low / scale_e) U_e^T into the product, the panel split
//               into hi and lo bf16 planes so that it keeps ~16 bits;
//   warps 2-3   idle;
//   warps 4-11  epilogue, two warps per TMEM lane quarter, each on half of the unit's columns: TMEM ->
//               registers, scale, bias, SwiGLU or its backward, bf16, global stores; the first four also turn the
//               panel into the bf16 operand of the last MMAs and store `low` for the backward pass.
// Two accumulators (columns 0 and 256 of a 512-column TMEM allocation) let the epilogue of one unit overlap
// the main loop of the next. Every barrier wait is bounded (common.cuh).
#include "common.cuh"
#include "host.hpp"

#ifndef MEEP2B_KSTEP_FENCE
#define MEEP2B_KSTEP_FENCE 1
#endif

namespace meep2b {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int BN = 192;
constexpr int RP = 16;  // rank panel width: the LoRA rank padded to 16
constexpr int A_BYTES = BM * BK * 2;      // 16 KB
constexpr int U_BYTES = BN * RP * 2;      // 6 KB
constexpr int LOW_BYTES = 2 * BM * RP * 2;  // 8 KB: the panel as two bf16 planes, hi and lo
constexpr int THREADS = 384;
constexpr int EPI_WARP0 = 4;
constexpr uint32_t TMEM_COLS = 512;
constexpr int ACC_STRIDE = 256;

// Shared-memory plan per mode. K-major: the B tile is 208 rows of 128 bytes; MN-major: four 64-column chunks.
// A staging area for the epilogue's TMA traffic: 8 warps x STG_BUFS tiles of 32 x 32 bf16. K-major and MN-major
// plain products keep 4 stages (4 KB and 2 KB of staging per warp); the MN-major dSwiGLU product keeps 3 (8 KB
// per warp: two buffers of a gate and an up tile, and their two load barriers per warp).
template <bool B_MN, int EPI = MEEP2B_EPI_PLAIN>
struct Plan {
  static constexpr bool DS = B_MN && EPI == MEEP2B_EPI_DSWIGLU;
  static constexpr int STAGES = 4;
  // per epilogue warp, in 2 KB buffers (the dSwiGLU epilogue: one 16-column chunk's gate and up tiles)
  static constexpr int STG_BUFS = DS ? 1 : (B_MN ? 1 : 2);
  static constexpr int B_BYTES = B_MN ? 4 * 64 * BK * 2 : (BN + RP) * BK * 2;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_U = OFF_B + STAGES * B_BYTES;
  static constexpr int OFF_LOW = OFF_U + U_BYTES;
  static constexpr int OFF_STG = OFF_LOW + LOW_BYTES;
  static constexpr int OFF_BAR = OFF_STG + 8 * STG_BUFS * 2048;
  static constexpr int NUM_BARS = 2 * STAGES + 10 + (DS ? 16 : 0);  // + the staged loads' barriers
  static constexpr int LD_BAR0 = 2 * STAGES + 10;                    // index of the first of those
  static constexpr int OFF_TMEM = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_TMEM + 16 + 1024;  // + slack to align the base to 1024
  static_assert(SMEM_BYTES <= 232448, "shared memory plan exceeds 227 KB");
  static_assert(B_BYTES % 1024 == 0 && OFF_U % 1024 == 0 && OFF_LOW % 1024 == 0 && OFF_STG % 1024 == 0,
                "swizzle atoms need 1 KB alignment");
};

struct Params {
  int rows, K, N, nblocks, kblocks, inter;
  int64_t ldo, ld_aux;
  const int32_t* offsets;
  const int32_t* tile_expert;
  const int32_t* tile_row;
  const int32_t* tiles;
  const float* scale;
  const __nv_bfloat16* bias;
  float scaling;
  __nv_bfloat16* out;
  __nv_bfloat16* low;
  __nv_bfloat16* aux;
  bool v8;  // out, aux and low rows 32-byte aligned: whole-sector stores
  // gathered x (GATHER kernels): tile row i is row a_rows[i] of the tensor the x map addresses
  const int32_t* a_rows;
  // dSwiGLU with the un-permute's backward folded in: the product is scaled by row_scale[row] (the routing weight)
  // and, when w_grad is set, w_grad[row * w_ld + block] = <unscaled product, h> over each 96-column block
  const float* row_scale;
  float* w_grad;
  int64_t w_ld;
  // PLAIN epilogue: product row i is stored at row out_rows[i] of out (token-major rows for a streaming combine)
  const int64_t* out_rows;
  bool staged;  // PLAIN epilogue: the out map exists, whole 32 x 32 tiles go out by TMA stores
};

// silu(g) = g / (1 + exp(-g)) with the fast exponential and division intrinsics; the result is rounded to bf16.
__device__ __forceinline__ float silu_f(float g) { return __fdividef(g, 1.0f + __expf(-g)); }
__device__ __forceinline__ float sigmoid_f(float g) { return __fdividef(1.0f, 1.0f + __expf(-g)); }

__device__ __forceinline__ void store32(__nv_bfloat16* dst, const uint32_t (&w)[16], int cnt) {
  if (cnt == 32) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int j = 0; j < 4; ++j) d4[j] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
  } else {
    for (int j = 0; j < cnt; ++j)
      dst[j] = __ushort_as_bfloat16(static_cast<unsigned short>(w[j >> 1] >> ((j & 1) * 16)));
  }
}

__device__ __forceinline__ void store16(__nv_bfloat16* dst, const uint32_t (&w)[8], int cnt) {
  if (cnt == 16) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
    d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
  } else {
    for (int j = 0; j < cnt; ++j)
      dst[j] = __ushort_as_bfloat16(static_cast<unsigned short>(w[j >> 1] >> ((j & 1) * 16)));
  }
}

// 32 bf16 of a row as 16 packed words; elements past cnt read as zero.
__device__ __forceinline__ void load32(const __nv_bfloat16* src, int cnt, uint32_t (&w)[16]) {
  if (cnt == 32) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 a = s4[j];
      w[4 * j] = a.x, w[4 * j + 1] = a.y, w[4 * j + 2] = a.z, w[4 * j + 3] = a.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t lo = 2 * j < cnt ? __bfloat16_as_ushort(src[2 * j]) : 0u;
      const uint32_t hi = 2 * j + 1 < cnt ? __bfloat16_as_ushort(src[2 * j + 1]) : 0u;
      w[j] = lo | (hi << 16);
    }
  }
}

// Arrival of an epilogue thread on a barrier of the MMA-issuing CTA: its own (one CTA per unit) or the pair
// leader's (rank 0 of a CTA pair).
template <bool PAIR>
__device__ __forceinline__ void arrive_on(uint32_t bar) {
  if (PAIR) {
    mbar_arrive_remote(bar, 0);
  } else {
    mbar_arrive(bar);
  }
}

// 16 bf16 (32 bytes, one DRAM sector) per store when the row is 32-byte aligned; 16-byte stores otherwise.
__device__ __forceinline__ void put16(__nv_bfloat16* dst, const uint32_t* w, bool v8) {
  if (v8) {
    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst), "r"(w[0]), "r"(w[1]),
                 "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
                 : "memory");
  } else {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
    d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
}

// cnt (<= 16) bf16 of w to dst: whole sectors when cnt == 16, element stores at a ragged edge.
__device__ __forceinline__ void put_n(__nv_bfloat16* dst, const uint32_t* w, int cnt, bool v8) {
  if (cnt == 16) {
    put16(dst, w, v8);
  } else {
    for (int j = 0; j < cnt; ++j)
      dst[j] = __ushort_as_bfloat16(static_cast<unsigned short>(w[j >> 1] >> ((j & 1) * 16)));
  }
}

// The 32 columns' raw accumulator words of this thread's row, issued without waiting (tcgen05.wait::ld joins).
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// tcgen05.wait::ld that also names the destination registers of the loads it completes, so that the compiler
// reads them only after the wait.
__device__ __forceinline__ void tmem_wait_regs16(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}

// One row of a 32-row x 16-column bf16 staging tile (32-byte rows with the 32-byte swizzle: the two 16-byte chunks
// of row r swap when bit 2 of r is set), written by the lane that owns the row: conflict-free 16-byte stores.
__device__ __forceinline__ void stage_row16(uint32_t tile, int lane, const uint32_t (&w)[8]) {
  const uint32_t r = tile + static_cast<uint32_t>(lane) * 32u;
  const uint32_t sw = (static_cast<uint32_t>(lane) >> 2) & 1u;
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(r + (sw << 4)), "r"(w[0]), "r"(w[1]), "r"(w[2]),
               "r"(w[3])
               : "memory");
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(r + ((sw ^ 1u) << 4)), "r"(w[4]), "r"(w[5]),
               "r"(w[6]), "r"(w[7])
               : "memory");
}

// The row `lane` of a 32-row x 16-column bf16 tile with the 32-byte swizzle (stage_row16's layout): 8 words, and
// the same row written back.
__device__ __forceinline__ void tile16_read(uint32_t tile, int lane, uint32_t (&w)[8]) {
  const uint32_t r = tile + static_cast<uint32_t>(lane) * 32u;
  const uint32_t sw = (static_cast<uint32_t>(lane) >> 2) & 1u;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
               : "r"(r + (sw << 4))
               : "memory");
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7])
               : "r"(r + ((sw ^ 1u) << 4))
               : "memory");
}

// A 32-row x 32-column bf16 tile in shared memory with the 64-byte swizzle (64-byte rows, the four 16-byte chunks
// of row r at chunk ^ ((r >> 1) & 3)): the lane that owns row `lane` reads or writes its 16 words.
__device__ __forceinline__ void tile32_read(uint32_t tile, int lane, uint32_t (&w)[16]) {
  const uint32_t r = tile + static_cast<uint32_t>(lane) * 64u;
  const uint32_t sw = (static_cast<uint32_t>(lane) >> 1) & 3u;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(w[4 * j]), "=r"(w[4 * j + 1]), "=r"(w[4 * j + 2]), "=r"(w[4 * j + 3])
                 : "r"(r + ((static_cast<uint32_t>(j) ^ sw) << 4))
                 : "memory");
}

__device__ __forceinline__ void tile32_write(uint32_t tile, int lane, const uint32_t (&w)[16]) {
  const uint32_t r = tile + static_cast<uint32_t>(lane) * 64u;
  const uint32_t sw = (static_cast<uint32_t>(lane) >> 1) & 3u;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(r + ((static_cast<uint32_t>(j) ^ sw) << 4)),
                 "r"(w[4 * j]), "r"(w[4 * j + 1]), "r"(w[4 * j + 2]), "r"(w[4 * j + 3])
                 : "memory");
}

// The dSwiGLU epilogue of one warp (32 rows, all of the expert, and `cols` <= 96 columns from n0) through shared
// memory, 16 columns at a time: the warp's lane 0 TMA-loads the chunk's gate and up pre-activation tiles (32 x 16
// each, 32-byte swizzle) into the warp's 2 KB buffer while the lanes read the chunk's accumulator words, every
// lane reads its row, writes dgate and dup over the tiles, and lane 0 TMA-stores them; the next chunk's tiles are
// loaded once the stores have read the buffer (one small buffer per warp, so that the operand ring keeps four
// stages). ldbar: the buffer's load barrier; phases: its next parity (bit 0).
template <bool PAIR>
__device__ __forceinline__ bool dswiglu_staged(const Params& p, int row0, int n0, int cols, float sc, float rw,
                                               uint32_t d, int lane, uint32_t stg, uint32_t ldbar, uint32_t& phases,
                                               const CUtensorMap* tm_aux, const CUtensorMap* tm_out,
                                               uint32_t bar_tfull_ab, uint32_t aph, uint32_t bar_tempty_ab,
                                               int64_t orow) {
  const int chunks = cols > 0 ? (cols + 15) / 16 : 0;
  if (chunks == 0) {
    if (!mbar_wait(bar_tfull_ab, aph)) return false;
    tc_fence_before();
    arrive_on<PAIR>(bar_tempty_ab);
    return true;
  }
  auto load = [&](int c) {
    if (lane == 0) {
      bulk_wait_read<0>();  // the buffer's last tiles have been read by their stores
      mbar_arrive_expect_tx(ldbar, 2048);
      tma_load_2d(stg, tm_aux, ldbar, n0 + 16 * c, row0);
      tma_load_2d(stg + 1024, tm_aux, ldbar, p.N + n0 + 16 * c, row0);
    }
  };
  load(0);
  if (!mbar_wait(bar_tfull_ab, aph)) return false;
  tc_fence_after();
  float wpart = 0.0f;
  bool ok = true;
  for (int c = 0; c < chunks; ++c) {
    uint32_t acc[16];
    tmem_ld16_async(d + 16 * c, acc);
    tmem_wait_regs16(acc);
    if (c + 1 == chunks) {
      tc_fence_before();
      arrive_on<PAIR>(bar_tempty_ab);  // the whole accumulator is in registers or done
    }
    if (!mbar_wait(ldbar, phases & 1u)) { ok = false; break; }
    phases ^= 1u;
    uint32_t gw[8], uw[8];
    tile16_read(stg, lane, gw);
    tile16_read(stg + 1024, lane, uw);
    const int cnt = min(16, cols - 16 * c);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float dgo[2], duo[2];
#pragma unroll
      for (int hlf = 0; hlf < 2; ++hlf) {
        const float gb = hlf ? bf16_hi(gw[j]) : bf16_lo(gw[j]);
        const float ub = hlf ? bf16_hi(uw[j]) : bf16_lo(uw[j]);
        const float dh_u = __uint_as_float(acc[2 * j + hlf]) * sc;
        const float dh = bf16_round(dh_u * rw);
        const float act = bf16_round(silu_f(gb));  // the forward's activation, bit for bit
        const float sig = sigmoid_f(gb);
        if (p.w_grad != nullptr && 2 * j + hlf < cnt) wpart += dh_u * bf16_round(act * ub);
        const float dact = bf16_round(dh * ub);
        duo[hlf] = dh * act;
        dgo[hlf] = dact * sig * (1.0f + gb * (1.0f - sig));
      }
      gw[j] = pack_bf16x2(dgo[0], dgo[1]);
      uw[j] = pack_bf16x2(duo[0], duo[1]);
    }
    stage_row16(stg, lane, gw);
    stage_row16(stg + 1024, lane, uw);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tm_out, stg, n0 + 16 * c, row0);
      tma_store_2d(tm_out, stg + 1024, p.N + n0 + 16 * c, row0);
      bulk_commit();
    }
    if (c + 1 < chunks) load(c + 1);
  }
  if (!ok) return false;
  if (p.w_grad != nullptr && cols > 0) p.w_grad[orow * p.w_ld + n0 / 96] = wpart;
  return true;
}

// The epilogue of one work unit for the 128 accumulator rows this CTA holds (TMEM lane quarter q, column half
// `half`). row_shift: the offset of this CTA's rows within the tile (128 for the second CTA of a pair). All of a
// thread's accumulator loads for the unit are issued before one wait (the dSwiGLU epilogue, which also reads the
// pre-activations, pipelines them by two). Returns false when a bounded wait ran out.
// SPLIT: the accumulator of an MN-major CTA pair, whose columns are [stack 0..95 | panel 0..7 | stack 96..191 |
// panel 8..15] (each CTA's half of B is 96 stack columns then 8 panel columns); otherwise [stack 0..191 | panel].
// stg / tm_out (plain epilogue): this warp's staging buffers in shared memory (stg_bufs of 2 KB, 1 KB-aligned) and
// the tensor map of `out` (boxes of 32 columns x 32 rows, 64-byte swizzle); when given, a warp whose 32 rows are
// all the expert's stores its columns as 32 x 32 tiles through shared memory with TMA stores (one bulk copy per
// tile instead of 32 rows of scattered 32-byte stores), and hands the accumulator back as soon as it is in
// registers. Rows at an expert's end (a warp with rows past it) and out_rows keep the per-row stores.
template <int EPI, bool LORA, bool PAIR, bool SPLIT = false>
__device__ __forceinline__ bool epilogue_unit(const Params& p, int u, int it, int row_shift, uint8_t* smem_low,
                                              uint32_t tmem_base, int q, int half, int lane,
                                              uint32_t bar_lowfull_ab, uint32_t bar_lowready,
                                              uint32_t bar_tfull_ab, uint32_t bar_tempty_ab, uint32_t stg = 0,
                                              const CUtensorMap* tm_out = nullptr, int stg_bufs = 0,
                                              const CUtensorMap* tm_aux = nullptr, uint32_t ldbar = 0,
                                              uint32_t* phases = nullptr) {
  const int r_in = q * 32 + lane;
  const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
  const int t = u / p.nblocks, nb = u - t * p.nblocks;
  const int e = p.tile_expert[t];
  const int row = p.tile_row[t] + row_shift + r_in;
  const bool valid = row < p.offsets[e];
  const int ab = it & 1;
  const uint32_t aph = (it >> 1) & 1;
  const float sc = p.scale != nullptr ? p.scale[e] : 1.0f;
  // the row's weight (the routing weight, when the un-permute's backward is folded in): scales the product row
  // and its stored rank panel; the adapter MMA's planes stay unscaled (the whole row is scaled at the end)
  const float rw = p.row_scale != nullptr && valid ? p.row_scale[row] : 1.0f;
  const uint32_t d = tmem_base + lane_base + ab * ACC_STRIDE;
  const int64_t orow = static_cast<int64_t>(row);
  const bool v8 = p.v8;
  if (LORA && half == 0) {
    if (!mbar_wait(bar_lowfull_ab, aph)) return false;
    tc_fence_after();
    float lv[16];
    if (SPLIT) {
      float l0[16], l1[16];
      tmem_ld16(d + 96, l0);    // panel columns 0..7 then stack columns 96..103 of the second half
      tmem_ld16(d + 200, l1);   // panel columns 8..15 then 8 columns past the tile
#pragma unroll
      for (int i = 0; i < 8; ++i) lv[i] = l0[i], lv[8 + i] = l1[i];
    } else {
      tmem_ld16(d + BN, lv);
    }
    if (p.low != nullptr && nb == 0 && valid) {
      uint32_t lw[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) lw[i] = pack_bf16x2(lv[2 * i] * rw, lv[2 * i + 1] * rw);
      put16(p.low + orow * RP, lw, v8);
    }
    // the A operand of the last MMAs: a = s * low / scale_e (float32) split into two bf16 planes, hi = bf16(a)
    // and lo = bf16(a - hi), K-major with the 32-byte swizzle (16-byte halves of a row swap on rows 4-7 of 8)
    const float f = p.scaling / sc;
    uint32_t hw[8], lo_w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float a0 = lv[2 * i] * f, a1 = lv[2 * i + 1] * f;
      hw[i] = pack_bf16x2(a0, a1);
      lo_w[i] = pack_bf16x2(a0 - bf16_lo(hw[i]), a1 - bf16_hi(hw[i]));
    }
    uint8_t* low_row = smem_low + r_in * 32;
    const int sw = (r_in >> 2) & 1;
    *reinterpret_cast<uint4*>(low_row + (0 ^ sw) * 16) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(low_row + (1 ^ sw) * 16) = make_uint4(hw[4], hw[5], hw[6], hw[7]);
    uint8_t* lo_row = low_row + BM * RP * 2;
    *reinterpret_cast<uint4*>(lo_row + (0 ^ sw) * 16) = make_uint4(lo_w[0], lo_w[1], lo_w[2], lo_w[3]);
    *reinterpret_cast<uint4*>(lo_row + (1 ^ sw) * 16) = make_uint4(lo_w[4], lo_w[5], lo_w[6], lo_w[7]);
    fence_proxy_async_smem();
    arrive_on<PAIR>(bar_lowready);
  }
  if (EPI == MEEP2B_EPI_SWIGLU) {
    // gate columns 0..95 and up columns 96..191 of the accumulator; this warp takes 48 of each
    const int n0h = nb * 96 + half * 48;
    const int cols = min(48, p.inter - n0h);
    uint32_t g[48], uu[48];
    if (!mbar_wait(bar_tfull_ab, aph)) return false;
    tc_fence_after();
    if (cols > 0) {
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        tmem_ld16_async(d + half * 48 + 16 * c, g + 16 * c);
        tmem_ld16_async(d + 96 + half * 48 + 16 * c, uu + 16 * c);
      }
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        tmem_wait_regs16(g + 16 * c);
        tmem_wait_regs16(uu + 16 * c);
      }
    }
    if (tm_out != nullptr && tm_aux != nullptr && p.staged && __all_sync(0xffffffffu, valid)) {
      // staged: per 16 columns the gate and up pre-activations and h as three 32 x 16 tiles, TMA-stored
      tc_fence_before();
      arrive_on<PAIR>(bar_tempty_ab);
      const __nv_bfloat16* bias_g = p.bias != nullptr ? p.bias + static_cast<int64_t>(e) * p.N + n0h : nullptr;
      const int row0 = p.tile_row[t] + row_shift + q * 32;
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        const int cnt = min(16, cols - 16 * c);
        if (cnt <= 0) break;
        uint32_t gw[8], uw[8], hw[8];
        const bool unit_scale = sc == 1.0f && rw == 1.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int k = 16 * c + 2 * j;
          float g0 = __uint_as_float(g[k]), g1 = __uint_as_float(g[k + 1]);
          float u0 = __uint_as_float(uu[k]), u1 = __uint_as_float(uu[k + 1]);
          if (!unit_scale) g0 = g0 * sc * rw, g1 = g1 * sc * rw, u0 = u0 * sc * rw, u1 = u1 * sc * rw;
          if (bias_g != nullptr && 2 * j + 1 < cnt) {
            g0 += __bfloat162float(bias_g[k]);
            g1 += __bfloat162float(bias_g[k + 1]);
            u0 += __bfloat162float(bias_g[p.inter + k]);
            u1 += __bfloat162float(bias_g[p.inter + k + 1]);
          }
          gw[j] = pack_bf16x2(g0, g1);
          uw[j] = pack_bf16x2(u0, u1);
          const uint32_t act = pack_bf16x2(silu_f(bf16_lo(gw[j])), silu_f(bf16_hi(gw[j])));  // bf16(silu(gate))
          hw[j] = pack_bf16x2(bf16_lo(act) * bf16_lo(uw[j]), bf16_hi(act) * bf16_hi(uw[j]));
        }
        if (lane == 0) bulk_wait_read<0>();  // the previous tiles have left the staging buffer
        __syncwarp();
        stage_row16(stg, lane, gw);
        stage_row16(stg + 1024, lane, uw);
        stage_row16(stg + 2048, lane, hw);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(tm_aux, stg, n0h + 16 * c, row0);
          tma_store_2d(tm_aux, stg + 1024, p.inter + n0h + 16 * c, row0);
          tma_store_2d(tm_out, stg + 2048, n0h + 16 * c, row0);
          bulk_commit();
        }
      }
      return true;
    }
    if (valid && cols > 0) {
      const __nv_bfloat16* bias_g = p.bias != nullptr ? p.bias + static_cast<int64_t>(e) * p.N + n0h : nullptr;
      __nv_bfloat16* pre = p.aux + orow * p.ld_aux + n0h;
      __nv_bfloat16* hrow = p.out + orow * p.ldo + n0h;
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        const int cnt = min(16, cols - 16 * c);
        if (cnt <= 0) break;
        uint32_t gw[8], uw[8], hw[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int k = 16 * c + 2 * j;
          float g0 = __uint_as_float(g[k]) * sc * rw, g1 = __uint_as_float(g[k + 1]) * sc * rw;
          float u0 = __uint_as_float(uu[k]) * sc * rw, u1 = __uint_as_float(uu[k + 1]) * sc * rw;
          if (bias_g != nullptr && 2 * j + 1 < cnt) {
            g0 += __bfloat162float(bias_g[k]);
            g1 += __bfloat162float(bias_g[k + 1]);
            u0 += __bfloat162float(bias_g[p.inter + k]);
            u1 += __bfloat162float(bias_g[p.inter + k + 1]);
          }
          gw[j] = pack_bf16x2(g0, g1);
          uw[j] = pack_bf16x2(u0, u1);
          const float a0 = bf16_round(silu_f(bf16_lo(gw[j]))), a1 = bf16_round(silu_f(bf16_hi(gw[j])));
          hw[j] = pack_bf16x2(a0 * bf16_lo(uw[j]), a1 * bf16_hi(uw[j]));
        }
        put_n(pre + 16 * c, gw, cnt, v8);
        put_n(pre + p.inter + 16 * c, uw, cnt, v8);
        put_n(hrow + 16 * c, hw, cnt, v8);
      }
    }
  } else if (EPI == MEEP2B_EPI_PLAIN) {
    constexpr int HS = SPLIT ? 104 : 96;  // accumulator column of the second half
    const int n0 = nb * BN + half * 96;
    const int cols = min(96, p.N - n0);
    uint32_t v[96];
    if (!mbar_wait(bar_tfull_ab, aph)) return false;
    tc_fence_after();
    if (cols > 0) {
      tmem_ld32_async(d + half * HS, *reinterpret_cast<uint32_t(*)[32]>(v));
      tmem_ld32_async(d + half * HS + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
      tmem_ld32_async(d + half * HS + 64, *reinterpret_cast<uint32_t(*)[32]>(v + 64));
#pragma unroll
      for (int c = 0; c < 6; ++c) tmem_wait_regs16(v + 16 * c);
    }
    if (tm_out != nullptr && p.staged && p.out_rows == nullptr && __all_sync(0xffffffffu, valid)) {
      tc_fence_before();
      arrive_on<PAIR>(bar_tempty_ab);  // the accumulator is in registers: the MMA may reuse it
      const __nv_bfloat16* bias = p.bias != nullptr ? p.bias + static_cast<int64_t>(e) * p.N + n0 : nullptr;
      const int row0 = p.tile_row[t] + row_shift + q * 32;
      if (lane == 0) bulk_wait_read<0>();  // the previous unit's tiles have left the staging buffers
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        if (cols - 32 * c <= 0) break;
        uint32_t w[16];
        const bool unit_scale = sc == 1.0f && rw == 1.0f;  // bf16 stacks without routing weights: no multiply
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int k = 32 * c + 2 * j;
          float a = __uint_as_float(v[k]), b = __uint_as_float(v[k + 1]);
          if (!unit_scale) a = a * sc * rw, b = b * sc * rw;
          if (bias != nullptr && 2 * j + 1 < cols - 32 * c) {
            a += __bfloat162float(bias[k]);
            b += __bfloat162float(bias[k + 1]);
          }
          w[j] = pack_bf16x2(a, b);
        }
        const uint32_t buf = stg + static_cast<uint32_t>(stg_bufs > 1 ? (c & 1) : 0) * 2048u;
        if (c >= stg_bufs) {  // the buffer's previous tile must have been read by its TMA store
          if (lane == 0) {
            if (stg_bufs > 1) bulk_wait_read<1>(); else bulk_wait_read<0>();
          }
          __syncwarp();
        }
        // row `lane`, 64 bytes, its four 16-byte chunks at chunk ^ ((row >> 1) & 3) (the 64-byte swizzle)
        const uint32_t rbase = buf + static_cast<uint32_t>(lane) * 64u;
        const uint32_t sw = (static_cast<uint32_t>(lane) >> 1) & 3u;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rbase + ((j ^ sw) << 4)), "r"(w[4 * j]),
                       "r"(w[4 * j + 1]), "r"(w[4 * j + 2]), "r"(w[4 * j + 3])
                       : "memory");
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(tm_out, buf, n0 + 32 * c, row0);
          bulk_commit();
        }
      }
      return true;
    }
    if (valid && cols > 0) {
      const __nv_bfloat16* bias = p.bias != nullptr ? p.bias + static_cast<int64_t>(e) * p.N + n0 : nullptr;
      const int64_t drow = p.out_rows != nullptr ? p.out_rows[row] : orow;
      __nv_bfloat16* dst = p.out + drow * p.ldo + n0;
#pragma unroll
      for (int c = 0; c < 6; ++c) {
        const int cnt = min(16, cols - 16 * c);
        if (cnt <= 0) break;
        uint32_t w[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int k = 16 * c + 2 * j;
          float a = __uint_as_float(v[k]) * sc * rw, b = __uint_as_float(v[k + 1]) * sc * rw;
          if (bias != nullptr && 2 * j + 1 < cnt) {
            a += __bfloat162float(bias[k]);
            b += __bfloat162float(bias[k + 1]);
          }
          w[j] = pack_bf16x2(a, b);
        }
        put_n(dst + 16 * c, w, cnt, v8);
      }
    }
  } else {  // MEEP2B_EPI_DSWIGLU: the product is dh; aux holds (gate, up); out receives (dgate, dup)
    // 16 columns per step, two steps in flight: the next step's accumulator words and pre-activations are
    // requested before this step is computed
    constexpr int HS = SPLIT ? 104 : 96;
    const int n0 = nb * BN + half * 96;
    const int cols = min(96, p.N - n0);
    if (tm_aux != nullptr && tm_out != nullptr && phases != nullptr && p.staged && __all_sync(0xffffffffu, valid))
      return dswiglu_staged<PAIR>(p, p.tile_row[t] + row_shift + q * 32, n0, cols, sc, rw, d + half * HS, lane, stg,
                                  ldbar, *phases, tm_aux, tm_out, bar_tfull_ab, aph, bar_tempty_ab, orow);
    const __nv_bfloat16* gp = p.aux + orow * p.ld_aux + n0;
    __nv_bfloat16* outp = p.out + orow * p.ldo + n0;
    uint32_t gw[2][8], uw[2][8], acc[2][16];
    auto load_pre = [&](int c, int b) {
      const int cnt = min(16, cols - 16 * c);
      if (cnt == 16) {
        const uint4 a0 = reinterpret_cast<const uint4*>(gp + 16 * c)[0], a1 = reinterpret_cast<const uint4*>(gp + 16 * c)[1];
        const uint4 b0 = reinterpret_cast<const uint4*>(gp + p.N + 16 * c)[0];
        const uint4 b1 = reinterpret_cast<const uint4*>(gp + p.N + 16 * c)[1];
        gw[b][0] = a0.x, gw[b][1] = a0.y, gw[b][2] = a0.z, gw[b][3] = a0.w;
        gw[b][4] = a1.x, gw[b][5] = a1.y, gw[b][6] = a1.z, gw[b][7] = a1.w;
        uw[b][0] = b0.x, uw[b][1] = b0.y, uw[b][2] = b0.z, uw[b][3] = b0.w;
        uw[b][4] = b1.x, uw[b][5] = b1.y, uw[b][6] = b1.z, uw[b][7] = b1.w;
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int k = 16 * c + 2 * j;
          const uint32_t g0 = 2 * j < cnt ? __bfloat16_as_ushort(gp[k]) : 0u;
          const uint32_t g1 = 2 * j + 1 < cnt ? __bfloat16_as_ushort(gp[k + 1]) : 0u;
          const uint32_t u0 = 2 * j < cnt ? __bfloat16_as_ushort(gp[p.N + k]) : 0u;
          const uint32_t u1 = 2 * j + 1 < cnt ? __bfloat16_as_ushort(gp[p.N + k + 1]) : 0u;
          gw[b][j] = g0 | (g1 << 16);
          uw[b][j] = u0 | (u1 << 16);
        }
      }
    };
    float wpart = 0.0f;  // <unscaled dh, h> over this thread's columns: the routing weight's gradient
    if (valid && cols > 0) load_pre(0, 0);
    if (!mbar_wait(bar_tfull_ab, aph)) return false;
    tc_fence_after();
    if (cols > 0) {
      tmem_ld16_async(d + half * HS, acc[0]);
      tmem_wait_regs16(acc[0]);
    }
#pragma unroll
    for (int c = 0; c < 6; ++c) {
      const int cnt = min(16, cols - 16 * c);
      if (cnt <= 0) break;
      const int b = c & 1;
      const bool more = c < 5 && cols - 16 * (c + 1) > 0;
      if (more) {
        tmem_ld16_async(d + half * HS + 16 * (c + 1), acc[b ^ 1]);
        if (valid) load_pre(c + 1, b ^ 1);
      }
      if (valid) {
        uint32_t dgw[8], duw[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float dgo[2], duo[2];
#pragma unroll
          for (int hlf = 0; hlf < 2; ++hlf) {
            const float gb = hlf ? bf16_hi(gw[b][j]) : bf16_lo(gw[b][j]);
            const float ub = hlf ? bf16_hi(uw[b][j]) : bf16_lo(uw[b][j]);
            const float dh_u = __uint_as_float(acc[b][2 * j + hlf]) * sc;
            const float dh = bf16_round(dh_u * rw);
            const float act = bf16_round(silu_f(gb));  // the forward's activation, bit for bit
            const float sig = sigmoid_f(gb);            // shares the exponential and reciprocal with silu_f
            if (p.w_grad != nullptr && 2 * j + hlf < cnt) wpart += dh_u * bf16_round(act * ub);  // h = bf16(act u)
            const float dact = bf16_round(dh * ub);
            duo[hlf] = dh * act;
            dgo[hlf] = dact * sig * (1.0f + gb * (1.0f - sig));
          }
          dgw[j] = pack_bf16x2(dgo[0], dgo[1]);
          duw[j] = pack_bf16x2(duo[0], duo[1]);
        }
        put_n(outp + 16 * c, dgw, cnt, v8);
        put_n(outp + p.N + 16 * c, duw, cnt, v8);
      }
      if (more) tmem_wait_regs16(acc[b ^ 1]);
    }
    if (p.w_grad != nullptr && valid && cols > 0) p.w_grad[orow * p.w_ld + n0 / 96] = wpart;
  }
  tc_fence_before();
  arrive_on<PAIR>(bar_tempty_ab);
  return true;
}

// Gathered x rows (products whose x rows are read where they are, from a token-major tensor through a_rows,
// without an expert-sorted copy): warp GATHER_WARP loads the x tile of every k-step by TMA gather4 loads (four rows
// of 64 columns each, at any rows of the source tensor), lane l taking tile rows 4 l .. 4 l + 3, into the x ring
// at a_ring (stage s at a_ring + s * A_BYTES) in the 128-byte-swizzled layout a tile load gives. The loads
// complete on the stage's full barrier (the pair leader's for a pair), whose bytes the producer announces with the
// stack's; a ring slot is refilled after its empty barrier completes. Tile rows past the product's end read row 0
// (the epilogue drops them).
constexpr int GATHER_WARP = 2;  // idle otherwise
template <int STAGES>
__device__ __forceinline__ void gather_role(const Params& p, const CUtensorMap* tm_src, int first_unit,
                                            int unit_stride, int total, int row_shift, uint32_t a_ring, uint32_t bar0,
                                            int lane, bool pair) {
  int stage = 0;
  uint32_t phase = 0;
  bool ok = true;
  for (int u = first_unit; u < total && ok; u += unit_stride) {
    const int t = u / p.nblocks;
    const int r = p.tile_row[t] + row_shift + 4 * lane;
    int src[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) src[j] = r + j < p.rows ? __ldg(p.a_rows + r + j) : 0;
    for (int kb = 0; kb < p.kblocks; ++kb) {
      ok = __all_sync(0xffffffffu, mbar_wait(bar0 + 8u * (STAGES + stage), phase ^ 1));
      if (!ok) break;
      const uint32_t dst = a_ring + stage * A_BYTES + lane * 512;
      if (pair) {
        tma_gather4_pair(dst, tm_src, map_to_rank(bar0 + 8u * stage, 0), kb * BK, src[0], src[1], src[2], src[3]);
      } else {
        tma_gather4(dst, tm_src, bar0 + 8u * stage, kb * BK, src[0], src[1], src[2], src[3]);
      }
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }
  }
  if (!ok) {
    // another role gave up after a bounded wait (its barrier may never complete): let this warp's last loads land
    // before the CTA's shared memory is released
    for (int i = 0; i < 64; ++i) __nanosleep(1000);
  }
}

template <bool B_MN, bool LORA, int EPI, bool GATHER = false>
__global__ void __launch_bounds__(THREADS, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                        const __grid_constant__ CUtensorMap tm_p, const __grid_constant__ CUtensorMap tm_u,
                        const __grid_constant__ CUtensorMap tm_out, const __grid_constant__ CUtensorMap tm_aux,
                        const Params p) {
  using P = Plan<B_MN, EPI>;
  constexpr int STAGES = P::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const uint32_t bar0 = sbase + P::OFF_BAR;
  auto bar_full = [&](int s) { return bar0 + 8u * s; };
  auto bar_empty = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto bar_tfull = [&](int b) { return bar0 + 8u * (2 * STAGES + b); };
  auto bar_tempty = [&](int b) { return bar0 + 8u * (2 * STAGES + 2 + b); };
  auto bar_lowfull = [&](int b) { return bar0 + 8u * (2 * STAGES + 4 + b); };
  const uint32_t bar_lowready = bar0 + 8u * (2 * STAGES + 6);
  const uint32_t bar_ufull = bar0 + 8u * (2 * STAGES + 7);
  const uint32_t bar_uempty = bar0 + 8u * (2 * STAGES + 8);
  const uint32_t bar_drain = bar0 + 8u * (2 * STAGES + 9);  // used only on the way out of a failed run
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + P::OFF_TMEM);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full(s), 1);
      mbar_init(bar_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_tfull(b), 1);
      mbar_init(bar_tempty(b), 256);
      mbar_init(bar_lowfull(b), 1);
    }
    mbar_init(bar_lowready, 128);
    mbar_init(bar_ufull, 1);
    mbar_init(bar_uempty, 1);
    mbar_init(bar_drain, 1);
    if (P::DS)
      for (int b = 0; b < 16; ++b) mbar_init(bar0 + 8u * (P::LD_BAR0 + b), 1);  // the epilogue's staged loads
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
    // (gathered x: the gather warp loads the x rows; this thread announces their bytes with the stack's)
    if (lane == 0) {
      const bool lead = true;
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_w);
      if (LORA) {
        tma_prefetch_desc(&tm_p);
        tma_prefetch_desc(&tm_u);
      }
      constexpr uint32_t B_TX = 64 * BN * 2 + (LORA ? (B_MN ? 64 * 64 * 2 : RP * 64 * 2) : 0);
      constexpr uint32_t STAGE_TX = A_BYTES + B_TX;
      auto wait = [&](uint32_t bar, uint32_t parity) -> bool { return mbar_wait(bar, parity); };
      int stage = 0;
      uint32_t phase = 0;
      uint32_t last_parity[STAGES];
      bool issued[STAGES];
      for (int s = 0; s < STAGES; ++s) issued[s] = false, last_parity[s] = 0;
      bool ok = true;
      int it = 0;
      // The up factor of a unit (single buffer) is loaded one k-step into the next unit, so that the producer never
      // waits for the previous unit's adapter MMAs while the ring could be refilled.
      int pu = -1, pu_nb = 0, pu_e = 0;
      auto load_u = [&]() -> bool {
        if (!wait(bar_uempty, (pu & 1) ^ 1)) return false;
        const uint32_t dst = sbase + P::OFF_U;
        if (lead) {
          mbar_arrive_expect_tx(bar_ufull, U_BYTES);
          if (!B_MN) {
            if (EPI == MEEP2B_EPI_SWIGLU) {
              tma_load_3d(dst, &tm_u, bar_ufull, 0, pu_nb * 96, pu_e);
              tma_load_3d(dst + 96 * RP * 2, &tm_u, bar_ufull, 0, p.inter + pu_nb * 96, pu_e);
            } else {
              tma_load_3d(dst, &tm_u, bar_ufull, 0, pu_nb * BN, pu_e);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 3; ++j) tma_load_3d(dst + j * 2048, &tm_u, bar_ufull, pu_nb * BN + 64 * j, 0, pu_e);
          }
        }
        pu = -1;
        return true;
      };
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ++it) {
        const int t = u / p.nblocks, nb = u - t * p.nblocks;
        const int e = p.tile_expert[t], row0 = p.tile_row[t];
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!wait(bar_empty(stage), phase ^ 1)) { ok = false; break; }
          const uint32_t fb = bar_full(stage);
          const uint32_t a_dst = sbase + P::OFF_A + stage * A_BYTES;
          const uint32_t b_dst = sbase + P::OFF_B + stage * P::B_BYTES;
          if (lead) {
            mbar_arrive_expect_tx(fb, STAGE_TX);
            if (!GATHER) tma_load_2d(a_dst, &tm_x, fb, kb * BK, row0);
            if (!B_MN) {
              if (EPI == MEEP2B_EPI_SWIGLU) {
                tma_load_3d(b_dst, &tm_w, fb, kb * BK, nb * 96, e);
                tma_load_3d(b_dst + 96 * 128, &tm_w, fb, kb * BK, p.inter + nb * 96, e);
              } else {
                tma_load_3d(b_dst, &tm_w, fb, kb * BK, nb * BN, e);
              }
              if (LORA) tma_load_3d(b_dst + BN * 128, &tm_p, fb, kb * BK, 0, e);
            } else {
#pragma unroll
              for (int j = 0; j < 3; ++j) tma_load_3d(b_dst + j * 8192, &tm_w, fb, nb * BN + 64 * j, kb * BK, e);
              if (LORA) tma_load_3d(b_dst + 3 * 8192, &tm_p, fb, 0, kb * BK, e);
            }
          }
          issued[stage] = true;
          last_parity[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
          if (LORA && kb == 0 && pu >= 0 && !load_u()) { ok = false; break; }
        }
        if (!ok) break;
        if (LORA) {
          if (pu >= 0 && !load_u()) { ok = false; break; }
          pu = it, pu_nb = nb, pu_e = e;
        }
      }
      if (ok && LORA && pu >= 0) ok = load_u();
      if (!ok && lead) {
        // a partner is gone: let this thread's copies in flight land before the CTA's shared memory goes away
        for (int s = 0; s < STAGES; ++s)
          if (issued[s]) mbar_wait_drain(bar_full(s), last_parity[s]);
      }
    }
  } else if (GATHER && warp == GATHER_WARP) {
    // ------------------------------------------------------------------------------------------ x-row gather
    gather_role<STAGES>(p, &tm_x, blockIdx.x, gridDim.x, total, 0, sbase + P::OFF_A, bar0, lane, false);
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_MAIN = idesc_bf16(BM, LORA ? BN + RP : BN, false, B_MN);
      constexpr uint32_t IDESC_UP = idesc_bf16(BM, BN, false, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      // The adapter MMAs of a unit wait for the epilogue to turn its panel into bf16 planes. Rather than idle
      // meanwhile, the issuer starts the next unit's main loop (in the other accumulator) and issues the pending
      // unit's adapter MMAs as soon as the panel is ready, tested between k-steps.
      int pend = -1;
      auto issue_up = [&](bool block) -> bool {
        const uint32_t par = static_cast<uint32_t>(pend) & 1;
        if (block) {
          if (!mbar_wait(bar_lowready, par) || !mbar_wait(bar_ufull, par)) return false;
        } else if (!mbar_test(bar_lowready, par) || !mbar_test(bar_ufull, par)) {
          return true;  // not yet: try again after the next k-step
        }
        tc_fence_after();
        const uint32_t dp = tmem_base + (pend & 1) * ACC_STRIDE;
        const uint32_t low_addr = sbase + P::OFF_LOW;
        const uint32_t u_addr = sbase + P::OFF_U;
        const uint64_t bdesc = B_MN ? smem_desc(u_addr, 2048, 1024, 2) : smem_desc(u_addr, 16, 256, 6);
        mma_bf16(dp, smem_desc(low_addr, 16, 256, 6), bdesc, IDESC_UP, 1);             // hi plane
        mma_bf16(dp, smem_desc(low_addr + BM * RP * 2, 16, 256, 6), bdesc, IDESC_UP, 1);  // lo plane
        mma_commit(bar_uempty);
        mma_commit(bar_tfull(pend & 1));
        pend = -1;
        return true;
      };
      // The descriptors of stage 0, k-slice 0; another stage or k-slice is an add to the start-address field
      // (bits 0-13, 16-byte units), which stays below 2^14 for every shared-memory address of the plan.
      const uint64_t a_desc0 = smem_desc(sbase + P::OFF_A, 16, 1024, 2);
      const uint64_t b_desc0 =
          B_MN ? smem_desc(sbase + P::OFF_B, 8192, 1024, 2) : smem_desc(sbase + P::OFF_B, 16, 1024, 2);
      constexpr uint32_t B_KK = B_MN ? 2048 / 16 : 32 / 16;  // one k-slice of 16, in 16-byte units
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ++it) {
        const int ab = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        if (!mbar_wait(bar_tempty(ab), aph ^ 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem_base + ab * ACC_STRIDE;
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait(bar_full(stage), phase)) { ok = false; break; }
          if (MEEP2B_KSTEP_FENCE) tc_fence_after();
          const uint64_t a_st = a_desc0 + static_cast<uint32_t>(stage) * (A_BYTES / 16);
          const uint64_t b_st = b_desc0 + static_cast<uint32_t>(stage) * (P::B_BYTES / 16);
          mma_bf16(d, a_st, b_st, IDESC_MAIN, kb != 0);
#pragma unroll
          for (int kk = 1; kk < BK / 16; ++kk) mma_bf16(d, a_st + 2 * kk, b_st + B_KK * kk, IDESC_MAIN, 1);
          mma_commit(bar_empty(stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
          if (LORA && pend >= 0 && !issue_up(false)) { ok = false; break; }
        }
        if (!ok) break;
        if (LORA) {
          if (pend >= 0 && !issue_up(true)) { ok = false; break; }
          mma_commit(bar_lowfull(ab));  // this unit's panel is in tensor memory: the epilogue may convert it
          pend = it;
        } else {
          mma_commit(bar_tfull(ab));
        }
      }
      if (ok && LORA && pend >= 0) ok = issue_up(true);
      if (!ok) {
        // let the MMAs already issued finish before tensor memory is released
        mma_commit(bar_drain);
        mbar_wait_drain(bar_drain, 0);
      }
    }
  } else if (warp >= EPI_WARP0) {
    // ------------------------------------------------------------------------------------------ epilogue
    const int q = warp & 3;                    // TMEM lane quarter this warp may read
    const int half = (warp - EPI_WARP0) >> 2;  // which half of the unit's columns
    int it = 0;
    const uint32_t stg = sbase + P::OFF_STG + static_cast<uint32_t>(warp - EPI_WARP0) * P::STG_BUFS * 2048u;
    const CUtensorMap* out_map = (EPI != MEEP2B_EPI_DSWIGLU || P::DS) ? &tm_out : nullptr;
    const CUtensorMap* aux_map = (EPI == MEEP2B_EPI_SWIGLU || P::DS) ? &tm_aux : nullptr;
    const uint32_t ldbar = bar0 + 8u * (P::LD_BAR0 + 2 * (warp - EPI_WARP0));
    uint32_t phases = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x, ++it) {
      const int ab = it & 1;
      if (!epilogue_unit<EPI, LORA, false>(p, u, it, 0, smem + P::OFF_LOW, tmem_base, q, half, lane, bar_lowfull(ab),
                                           bar_lowready, bar_tfull(ab), bar_tempty(ab), stg, out_map, P::STG_BUFS,
                                           aux_map, ldbar, P::DS ? &phases : nullptr))
        break;
    }
    if (lane == 0) bulk_wait_all();  // this warp's TMA stores are done before the CTA's shared memory goes away
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// CTA-pair variant (tcgen05 cta_group::2) for stacks read K-major. A work unit is 256 rows of one expert by 192
// columns. CTA r of the pair loads rows 128r..128r+127 of the x tile and rows 104r..104r+103 of the 208-row B tile
// (the 192 stack rows, then the 16 panel rows), so each SM stages half of B; the pair leader issues M=256 N=208
// MMAs that write both CTAs' tensor memory (each holds its 128 rows of the 208 columns). The epilogue is the
// same per CTA. All loads are plain TMA tile loads into the loading CTA's own shared memory, completing on the
// leader's barrier; there is no multicast.
#ifndef MEEP2B_PAIR_STAGES
#define MEEP2B_PAIR_STAGES 6
#endif
constexpr int PAIR_STAGES = MEEP2B_PAIR_STAGES;
constexpr int PAIR_B_ROWS = (BN + RP) / 2;  // 104: each CTA's share of the 208 K-major B rows

// Shared memory of a CTA of a pair. K-major: per stage the x tile and 104 B rows (7 stages). MN-major: the x tile,
// then this CTA's 96 stack columns as three 32-column atoms with the 64-byte swizzle (64 rows x 64 B each) and,
// right after them, a fourth atom whose first 8 columns are its 8 panel columns: the 104 columns the pair's N = 208
// MMA reads from it (6 stages).
template <bool B_MN>
struct PairPlan {
  static constexpr int STAGES = B_MN ? 5 : PAIR_STAGES;
  static constexpr int B_BYTES = B_MN ? 4 * 64 * 64 : PAIR_B_ROWS * BK * 2;  // 16 KB : 13 KB
  static constexpr int PANEL_OFF = 3 * 64 * 64;                            // MN-major panel atom
  static constexpr int U_TX = B_MN ? 4 * RP * 64 : (BN / 2) * RP * 2;      // bytes of U each CTA loads
  static constexpr int U_BYTES = 4096;
  static constexpr int OFF_B = STAGES * A_BYTES;
  static constexpr int OFF_U = OFF_B + STAGES * B_BYTES;
  static constexpr int OFF_LOW = OFF_U + U_BYTES;
  static constexpr int STG_BUFS = 2;  // 4 KB of staging per epilogue warp (two 32 x 32 tiles, or three 32 x 16)
  static constexpr int OFF_STG = OFF_LOW + LOW_BYTES;
  static constexpr int OFF_BAR = OFF_STG + 8 * STG_BUFS * 2048;
  static constexpr int NUM_BARS = 2 * STAGES + 10;
  static constexpr int OFF_TMEM = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_TMEM + 16 + 1024;
  static_assert(SMEM_BYTES <= 232448, "pair shared memory plan exceeds 227 KB");
  static_assert(B_BYTES % 1024 == 0 && OFF_U % 1024 == 0 && OFF_LOW % 1024 == 0, "1 KB alignment");
};

struct PairMaps {
  CUtensorMap x;     // (k, rows) box 64 x 128
  CUtensorMap w104;  // (k, n, E) box 64 x 104
  CUtensorMap w96;   // box 64 x 96
  CUtensorMap w88;   // box 64 x 88
  CUtensorMap w8;    // box 64 x 8
  CUtensorMap p16;   // panel (k, 16, E) box 64 x 16
  CUtensorMap u96;   // up (16, n, E) box 16 x 96, 32-byte swizzle
  CUtensorMap w_mn;  // MN-major stack (n, k, E) box 32 x 64, 64-byte swizzle
  CUtensorMap p_mn;  // MN-major panel (E, k, 64) box 32 x 64 from column 8 * rank, 64-byte swizzle
  CUtensorMap u_mn;  // MN-major up factor (n, 16, E) box 32 x 16, 64-byte swizzle
  CUtensorMap out;   // the epilogue's TMA stores (as the one-CTA kernel's tm_out)
  CUtensorMap aux;   // SwiGLU pre-activations (as tm_aux)
};

template <bool B_MN, bool LORA, int EPI, bool GATHER = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    grouped_gemm_pair_kernel(const __grid_constant__ PairMaps m, const Params p) {
  using PP = PairPlan<B_MN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair_id = static_cast<int>(cluster_id_x()), pairs = static_cast<int>(num_clusters_x());

  const uint32_t bar0 = sbase + PP::OFF_BAR;
  auto bar_full = [&](int s) { return bar0 + 8u * s; };
  auto bar_empty = [&](int s) { return bar0 + 8u * (PP::STAGES + s); };
  auto bar_tfull = [&](int b) { return bar0 + 8u * (2 * PP::STAGES + b); };
  auto bar_tempty = [&](int b) { return bar0 + 8u * (2 * PP::STAGES + 2 + b); };
  auto bar_lowfull = [&](int b) { return bar0 + 8u * (2 * PP::STAGES + 4 + b); };
  const uint32_t bar_lowready = bar0 + 8u * (2 * PP::STAGES + 6);
  const uint32_t bar_ufull = bar0 + 8u * (2 * PP::STAGES + 7);
  const uint32_t bar_uempty = bar0 + 8u * (2 * PP::STAGES + 8);
  const uint32_t bar_drain = bar0 + 8u * (2 * PP::STAGES + 9);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + PP::OFF_TMEM);

  if (threadIdx.x == 0) {
    for (int s = 0; s < PP::STAGES; ++s) {
      mbar_init(bar_full(s), 1);
      mbar_init(bar_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_tfull(b), 1);
      mbar_init(bar_tempty(b), 512);  // 256 epilogue threads of each CTA
      mbar_init(bar_lowfull(b), 1);
    }
    mbar_init(bar_lowready, 256);  // 128 per CTA
    mbar_init(bar_ufull, 1);
    mbar_init(bar_uempty, 1);
    mbar_init(bar_drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrival or load
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total = (*p.tiles) * p.nblocks;

  if (warp == 0) {
    // ------------------------------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const bool lead = true;
      tma_prefetch_desc(&m.x);
      // K-major: with the panel the 208 B rows split 104 / 104 (the second CTA's last 16 are the panel), without it
      // 96 / 96. MN-major: 96 stack columns per CTA, plus 8 panel columns (one 16-column atom) with the adapters.
      constexpr uint32_t CTA_TX =
          A_BYTES + (B_MN ? 3 * 64 * 64 + (LORA ? 64 * 64 : 0) : (LORA ? PAIR_B_ROWS : BN / 2) * 128);
      auto wait = [&](uint32_t bar, uint32_t parity) -> bool { return mbar_wait(bar, parity); };
      int stage = 0;
      uint32_t phase = 0;
      uint32_t last_parity[PP::STAGES];
      bool issued[PP::STAGES];
      for (int s = 0; s < PP::STAGES; ++s) issued[s] = false, last_parity[s] = 0;
      bool ok = true;
      int it = 0;
      int pu = -1, pu_nb = 0, pu_e = 0;  // as in the one-CTA kernel: a unit's up factor goes out one k-step later
      auto load_u = [&]() -> bool {
        if (!wait(bar_uempty, (pu & 1) ^ 1)) return false;
        if (lead) {
          if (rank == 0) mbar_arrive_expect_tx(bar_ufull, 2 * PP::U_TX);
          const int urow = EPI == MEEP2B_EPI_SWIGLU ? (rank == 0 ? pu_nb * 96 : p.inter + pu_nb * 96)
                                                    : pu_nb * BN + 96 * static_cast<int>(rank);
          if (B_MN) {  // 96 columns and 8 more: the fourth atom lands on panel columns of the accumulator, read already
#pragma unroll
            for (int j = 0; j < 4; ++j)
              tma_load_3d_pair(sbase + PP::OFF_U + j * 1024, &m.u_mn, map_to_rank(bar_ufull, 0), urow + 32 * j, 0, pu_e);
          } else {
            tma_load_3d_pair(sbase + PP::OFF_U, &m.u96, map_to_rank(bar_ufull, 0), 0, urow, pu_e);
          }
        }
        pu = -1;
        return true;
      };
      for (int u = pair_id; u < total && ok; u += pairs, ++it) {
        const int t = u / p.nblocks, nb = u - t * p.nblocks;
        const int e = p.tile_expert[t], row0 = p.tile_row[t] + 128 * static_cast<int>(rank);
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!wait(bar_empty(stage), phase ^ 1)) { ok = false; break; }
          const uint32_t fb = bar_full(stage);
          const uint32_t fb_lead = map_to_rank(fb, 0);
          const uint32_t a_dst = sbase + stage * A_BYTES;
          const uint32_t b_dst = sbase + PP::OFF_B + stage * PP::B_BYTES;
          const int k0 = kb * BK;
          if (lead) {
            if (rank == 0) mbar_arrive_expect_tx(fb, 2 * CTA_TX);
            if (!GATHER) tma_load_2d_pair(a_dst, &m.x, fb_lead, kb * BK, row0);
            if (B_MN) {
              const int c0 = nb * BN + 96 * static_cast<int>(rank);
#pragma unroll
              for (int j = 0; j < 3; ++j) tma_load_3d_pair(b_dst + j * 4096, &m.w_mn, fb_lead, c0 + 32 * j, k0, e);
              if (LORA) tma_load_3d_pair(b_dst + PP::PANEL_OFF, &m.p_mn, fb_lead, 8 * static_cast<int>(rank), k0, e);
            } else if (EPI == MEEP2B_EPI_SWIGLU) {
              const int g0 = nb * 96;
              if (!LORA) {  // gate rows in the first CTA, up rows in the second
                tma_load_3d_pair(b_dst, &m.w96, fb_lead, k0, rank == 0 ? g0 : p.inter + g0, e);
              } else if (rank == 0) {
                tma_load_3d_pair(b_dst, &m.w96, fb_lead, k0, g0, e);                       // gate 0..95
                tma_load_3d_pair(b_dst + 96 * 128, &m.w8, fb_lead, k0, p.inter + g0, e);   // up 0..7
              } else {
                tma_load_3d_pair(b_dst, &m.w88, fb_lead, k0, p.inter + g0 + 8, e);         // up 8..95
                tma_load_3d_pair(b_dst + 88 * 128, &m.p16, fb_lead, k0, 0, e);             // the rank panel
              }
            } else {
              const int n0 = nb * BN;
              if (!LORA) {
                tma_load_3d_pair(b_dst, &m.w96, fb_lead, k0, n0 + 96 * static_cast<int>(rank), e);
              } else if (rank == 0) {
                tma_load_3d_pair(b_dst, &m.w104, fb_lead, k0, n0, e);
              } else {
                tma_load_3d_pair(b_dst, &m.w88, fb_lead, k0, n0 + 104, e);
                tma_load_3d_pair(b_dst + 88 * 128, &m.p16, fb_lead, k0, 0, e);             // the rank panel
              }
            }
          }
          issued[stage] = true;
          last_parity[stage] = phase;
          if (++stage == PP::STAGES) {
            stage = 0;
            phase ^= 1;
          }
          if (LORA && kb == 0 && pu >= 0 && !load_u()) { ok = false; break; }
        }
        if (!ok) break;
        if (LORA) {
          if (pu >= 0 && !load_u()) { ok = false; break; }
          pu = it, pu_nb = nb, pu_e = e;
        }
      }
      if (ok && LORA && pu >= 0) ok = load_u();
      if (!ok && lead) {
        for (int s = 0; s < PP::STAGES; ++s)
          if (issued[s] && rank == 0) mbar_wait_drain(bar_full(s), last_parity[s]);
      }
    }
  } else if (GATHER && warp == GATHER_WARP) {
    // ------------------------------------------------------------------------------------------ x-row gather
    gather_role<PP::STAGES>(p, &m.x, pair_id, pairs, total, 128 * static_cast<int>(rank), sbase, bar0, lane, true);
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------------------ MMA issuer (leader)
    if (lane == 0 && rank == 0) {
      // one MMA of N = 208 with the adapters (the panel rides along in the B tile), 192 without; the MN-major
      // adapter MMA also spans 208 columns so that its two halves land on the split accumulator's stack columns
      constexpr uint32_t IDESC_MAIN = idesc_bf16(256, LORA ? BN + RP : BN, false, B_MN);
      constexpr uint32_t IDESC_UP = idesc_bf16(256, B_MN ? BN + RP : BN, false, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      int pend = -1;  // as in the one-CTA kernel: a unit's adapter MMAs go out during the next unit's main loop
      auto issue_up = [&](bool block) -> bool {
        const uint32_t par = static_cast<uint32_t>(pend) & 1;
        if (block) {
          if (!mbar_wait_cluster(bar_lowready, par) || !mbar_wait(bar_ufull, par)) return false;
        } else if (!mbar_test_cluster(bar_lowready, par) || !mbar_test(bar_ufull, par)) {
          return true;
        }
        tc_fence_after();
        const uint32_t dp = tmem_base + (pend & 1) * ACC_STRIDE;
        const uint32_t low_addr = sbase + PP::OFF_LOW;
        const uint64_t bdesc =
            B_MN ? smem_desc(sbase + PP::OFF_U, 1024, 512, 4) : smem_desc(sbase + PP::OFF_U, 16, 256, 6);
        mma_bf16_pair(dp, smem_desc(low_addr, 16, 256, 6), bdesc, IDESC_UP, 1);             // hi plane
        mma_bf16_pair(dp, smem_desc(low_addr + BM * RP * 2, 16, 256, 6), bdesc, IDESC_UP, 1);  // lo plane
        mma_commit_pair(bar_uempty);
        mma_commit_pair(bar_tfull(pend & 1));
        pend = -1;
        return true;
      };
      // descriptors of stage 0, k-slice 0, advanced by adds to the start-address field (as in the one-CTA kernel)
      const uint64_t a_desc0 = smem_desc(sbase, 16, 1024, 2);
      const uint64_t b_desc0 =
          B_MN ? smem_desc(sbase + PP::OFF_B, 4096, 512, 4) : smem_desc(sbase + PP::OFF_B, 16, 1024, 2);
      constexpr uint32_t B_KK = B_MN ? 1024 / 16 : 32 / 16;
      for (int u = pair_id; u < total && ok; u += pairs, ++it) {
        const int ab = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        if (!mbar_wait_cluster(bar_tempty(ab), aph ^ 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem_base + ab * ACC_STRIDE;
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait(bar_full(stage), phase)) {
            ok = false;
            break;
          }
          if (MEEP2B_KSTEP_FENCE) tc_fence_after();
          const uint64_t a_st = a_desc0 + static_cast<uint32_t>(stage) * (A_BYTES / 16);
          const uint64_t b_st = b_desc0 + static_cast<uint32_t>(stage) * (PP::B_BYTES / 16);
          mma_bf16_pair(d, a_st, b_st, IDESC_MAIN, kb != 0);
#pragma unroll
          for (int kk = 1; kk < BK / 16; ++kk) mma_bf16_pair(d, a_st + 2 * kk, b_st + B_KK * kk, IDESC_MAIN, 1);
          mma_commit_pair(bar_empty(stage));
          if (++stage == PP::STAGES) {
            stage = 0;
            phase ^= 1;
          }
          if (LORA && pend >= 0 && !issue_up(false)) { ok = false; break; }
        }
        if (!ok) break;
        if (LORA) {
          if (pend >= 0 && !issue_up(true)) { ok = false; break; }
          mma_commit_pair(bar_lowfull(ab));
          pend = it;
        } else {
          mma_commit_pair(bar_tfull(ab));
        }
      }
      if (ok && LORA && pend >= 0) ok = issue_up(true);
      if (!ok) {
        mma_commit_pair(bar_drain);
        mbar_wait_drain(bar_drain, 0);
      }
    }
  } else if (warp >= EPI_WARP0) {
    // ------------------------------------------------------------------------------------------ epilogue (each CTA)
    const int q = warp & 3;
    const int half = (warp - EPI_WARP0) >> 2;
    int it = 0;
    const uint32_t stg = sbase + PP::OFF_STG + static_cast<uint32_t>(warp - EPI_WARP0) * PP::STG_BUFS * 2048u;
    const CUtensorMap* out_map = EPI != MEEP2B_EPI_DSWIGLU ? &m.out : nullptr;
    const CUtensorMap* aux_map = EPI == MEEP2B_EPI_SWIGLU ? &m.aux : nullptr;
    for (int u = pair_id; u < total; u += pairs, ++it) {
      const int ab = it & 1;
      if (!epilogue_unit<EPI, LORA, true, B_MN && LORA>(p, u, it, 128 * static_cast<int>(rank), smem + PP::OFF_LOW,
                                                        tmem_base, q, half, lane, bar_lowfull(ab), bar_lowready,
                                                        bar_tfull(ab), bar_tempty(ab), stg, out_map, PP::STG_BUFS,
                                                        aux_map))
        break;
    }
    if (lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  cluster_sync();  // no CTA releases tensor memory while the pair's MMAs or the other epilogue may still use it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

template <bool B_MN, bool LORA, int EPI, bool GATHER = false>
static int launch_pair(const PairMaps& maps, const Params& prm, int grid, cudaStream_t s) {
  auto kern = grouped_gemm_pair_kernel<B_MN, LORA, EPI, GATHER>;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PairPlan<B_MN>::SMEM_BYTES) != cudaSuccess) {
      cudaGetLastError();
      return MEEP2B_ERR_LAUNCH;
    }
    configured = true;
  }
  kern<<<grid, THREADS, PairPlan<B_MN>::SMEM_BYTES, s>>>(maps, prm);
  return launch_status();
}

template <bool B_MN, bool LORA, int EPI, bool GATHER = false>
static int launch(const CUtensorMap& tx, const CUtensorMap& tw, const CUtensorMap& tp, const CUtensorMap& tu,
                  const CUtensorMap& tout, const CUtensorMap& taux, const Params& prm, int grid, cudaStream_t s) {
  auto kern = grouped_gemm_kernel<B_MN, LORA, EPI, GATHER>;
  static bool configured = false;  // per instantiation; attributes are per device but idempotent
  if (!configured) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Plan<B_MN, EPI>::SMEM_BYTES) != cudaSuccess) {
      cudaGetLastError();
      return MEEP2B_ERR_LAUNCH;
    }
    configured = true;
  }
  kern<<<grid, THREADS, Plan<B_MN, EPI>::SMEM_BYTES, s>>>(tx, tw, tp, tu, tout, taux, prm);
  return launch_status();
}

#include "grouped_gemm_q.cuh"
#include "grouped_gemm_qpair.cuh"

}  // namespace gemm
}  // namespace meep2b

using namespace meep2b;
using namespace meep2b::gemm;

extern "C" int meep2b_grouped_product(const meep2b_product* a, void* stream) {
  if (a == nullptr) return MEEP2B_ERR_SHAPE;
  const bool quantised = a->weight_dtype == MEEP2B_NF4 || a->weight_dtype == MEEP2B_E4M3 ||
                         a->weight_dtype == MEEP2B_E4M3_BLOCKS;
  if (a->weight_dtype != MEEP2B_BF16 && !quantised) return MEEP2B_ERR_UNSUPPORTED;
  if (quantised && a->block_m == 256 && a->b_mn) return MEEP2B_ERR_UNSUPPORTED;  // quantised pairs: K-major only
  if (a->rows < 0 || a->k < 1 || a->n < 1 || a->experts < 1) return MEEP2B_ERR_SHAPE;
  if (a->k % 8 || a->n % 8 || a->ldx % 8 || a->ldo % 8 || a->ldx < a->k) return MEEP2B_ERR_ALIGN;
  if (a->rows > INT32_MAX || a->k > INT32_MAX || a->n > INT32_MAX) return MEEP2B_ERR_SHAPE;
  const bool lora = a->panel != nullptr;
  if (lora && a->up == nullptr) return MEEP2B_ERR_SHAPE;
  const int epi = a->epilogue;
  if (epi < MEEP2B_EPI_PLAIN || epi > MEEP2B_EPI_DSWIGLU) return MEEP2B_ERR_UNSUPPORTED;
  if (epi == MEEP2B_EPI_SWIGLU && (a->b_mn || a->n % 16)) return MEEP2B_ERR_UNSUPPORTED;
  if (epi != MEEP2B_EPI_PLAIN && a->aux == nullptr) return MEEP2B_ERR_SHAPE;
  if (!aligned16(a->x) || !aligned16(a->weight) || !aligned16(a->out) || (a->low && !aligned16(a->low)) ||
      (a->aux && !aligned16(a->aux)) || (lora && (!aligned16(a->panel) || !aligned16(a->up))))
    return MEEP2B_ERR_ALIGN;
  const bool gather = a->x_rows != nullptr;
  if (gather && (quantised || a->x_src_rows < 1 ||
                 !((epi == MEEP2B_EPI_SWIGLU && !a->b_mn) || (epi == MEEP2B_EPI_DSWIGLU && a->b_mn))))
    return MEEP2B_ERR_UNSUPPORTED;
  if (a->w_grad != nullptr && (epi != MEEP2B_EPI_DSWIGLU || a->w_ld < (a->n + 95) / 96)) return MEEP2B_ERR_SHAPE;
  if (a->out_rows != nullptr && (epi != MEEP2B_EPI_PLAIN || quantised)) return MEEP2B_ERR_UNSUPPORTED;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  if (a->rows == 0) return MEEP2B_OK;

  const uint64_t K = a->k, N = a->n, E = a->experts, rows = a->rows;
  const uint64_t x_rows_in_map = gather ? static_cast<uint64_t>(a->x_src_rows) : rows;
  CUtensorMap tx, tw, tp, tu, tout, taux;
  // The epilogue's TMA stores (bf16 stacks): the plain epilogue's out map in 32 x 32 boxes (64-byte swizzle); the
  // SwiGLU epilogue's h (out) and pre-activation (aux) maps in 16-column x 32-row boxes (32-byte swizzle), when the
  // gate and up halves are whole 16-column tiles.
  bool staged = false;
  if (epi == MEEP2B_EPI_PLAIN && !quantised && a->out_rows == nullptr && a->n >= 32 && a->rows >= 32) {
    const uint64_t od[2] = {static_cast<uint64_t>(a->n), static_cast<uint64_t>(a->rows)};
    const uint64_t os[1] = {static_cast<uint64_t>(a->ldo) * 2};
    const uint32_t ob[2] = {32, 32};
    staged = encode_tiled(&tout, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a->out, od, os, ob,
                          CU_TENSOR_MAP_SWIZZLE_64B) == MEEP2B_OK;
  } else if (epi == MEEP2B_EPI_DSWIGLU && !quantised && a->b_mn && a->block_m != 256 && a->n % 16 == 0 &&
             a->rows >= 32) {
    // the dSwiGLU epilogue's pre-activation loads and gradient stores: (rows, 2n) maps in 16-column x 32-row boxes
    const uint64_t od[2] = {static_cast<uint64_t>(2 * a->n), static_cast<uint64_t>(a->rows)};
    const uint64_t os[1] = {static_cast<uint64_t>(a->ldo) * 2};
    const uint64_t as[1] = {static_cast<uint64_t>(2 * a->n) * 2};
    const uint32_t bx[2] = {16, 32};
    staged = encode_tiled(&tout, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a->out, od, os, bx,
                          CU_TENSOR_MAP_SWIZZLE_32B) == MEEP2B_OK &&
             encode_tiled(&taux, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a->aux, od, as, bx,
                          CU_TENSOR_MAP_SWIZZLE_32B) == MEEP2B_OK;
  } else if (epi == MEEP2B_EPI_SWIGLU && !quantised && (a->n / 2) % 16 == 0 && a->rows >= 32) {
    const uint64_t od[2] = {static_cast<uint64_t>(a->n / 2), static_cast<uint64_t>(a->rows)};
    const uint64_t os[1] = {static_cast<uint64_t>(a->ldo) * 2};
    const uint64_t ad[2] = {static_cast<uint64_t>(a->n), static_cast<uint64_t>(a->rows)};
    const uint64_t as[1] = {static_cast<uint64_t>(a->n) * 2};
    const uint32_t bx[2] = {16, 32};
    staged = encode_tiled(&tout, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a->out, od, os, bx,
                          CU_TENSOR_MAP_SWIZZLE_32B) == MEEP2B_OK &&
             encode_tiled(&taux, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a->aux, ad, as, bx,
                          CU_TENSOR_MAP_SWIZZLE_32B) == MEEP2B_OK;
  }
  {
    const uint64_t dims[2] = {K, x_rows_in_map};
    const uint64_t strides[1] = {static_cast<uint64_t>(a->ldx) * 2};
    const uint32_t box[2] = {64, gather ? 1u : 128u};  // gathered rows: tile::gather4 loads, one-row boxes
    MEEP2B_TRY(encode_tiled(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a->x, dims, strides, box,
                            CU_TENSOR_MAP_SWIZZLE_128B));
  }
  const uint32_t rows_per_load = (epi == MEEP2B_EPI_SWIGLU) ? 96 : BN;
  if (quantised) {
    tw = tx;  // the codes get their own map (launch_quantized)
  } else if (!a->b_mn) {
    const uint64_t dims[3] = {K, N, E};
    const uint64_t strides[2] = {K * 2, N * K * 2};
    const uint32_t box[3] = {64, rows_per_load, 1};
    MEEP2B_TRY(encode_tiled(&tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a->weight, dims, strides, box,
                            CU_TENSOR_MAP_SWIZZLE_128B));
  } else {
    const uint64_t dims[3] = {N, K, E};
    const uint64_t strides[2] = {N * 2, K * N * 2};
    const uint32_t box[3] = {64, 64, 1};
    MEEP2B_TRY(encode_tiled(&tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a->weight, dims, strides, box,
                            CU_TENSOR_MAP_SWIZZLE_128B));
  }
  if (lora) {
    if (!a->b_mn) {
      const uint64_t pd[3] = {K, RP, E};
      const uint64_t ps[2] = {K * 2, RP * K * 2};
      const uint32_t pb[3] = {64, RP, 1};
      MEEP2B_TRY(encode_tiled(&tp, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a->panel, pd, ps, pb,
                              CU_TENSOR_MAP_SWIZZLE_128B));
      const uint64_t ud[3] = {RP, N, E};
      const uint64_t us[2] = {RP * 2, N * RP * 2};
      const uint32_t ubx[3] = {RP, rows_per_load, 1};
      MEEP2B_TRY(encode_tiled(&tu, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a->up, ud, us, ubx,
                              CU_TENSOR_MAP_SWIZZLE_32B));
    } else {
      // the (E, k, 16) panel read as 64-column boxes: the 48 columns past its width arrive as zeros (the box's
      // out-of-bounds fill), the panel atom of the MN-major B tile
      const uint64_t pd[3] = {RP, K, E};
      const uint64_t ps[2] = {RP * 2, K * RP * 2};
      const uint32_t pb[3] = {64, 64, 1};
      MEEP2B_TRY(encode_tiled(&tp, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a->panel, pd, ps, pb,
                              CU_TENSOR_MAP_SWIZZLE_128B));
      const uint64_t ud[3] = {N, RP, E};
      const uint64_t us[2] = {N * 2, RP * N * 2};
      const uint32_t ubx[3] = {64, RP, 1};
      MEEP2B_TRY(encode_tiled(&tu, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a->up, ud, us, ubx,
                              CU_TENSOR_MAP_SWIZZLE_128B));
    }
  } else {
    tp = tx;
    tu = tx;
  }

  Params prm;
  prm.rows = static_cast<int>(rows);
  prm.K = static_cast<int>(K);
  prm.N = static_cast<int>(N);
  prm.inter = (epi == MEEP2B_EPI_SWIGLU) ? static_cast<int>(N / 2) : static_cast<int>(N);
  prm.nblocks = (epi == MEEP2B_EPI_SWIGLU) ? (prm.inter + 95) / 96 : static_cast<int>((N + BN - 1) / BN);
  prm.kblocks = static_cast<int>((K + BK - 1) / BK);
  prm.ldo = a->ldo;
  prm.ld_aux = (epi == MEEP2B_EPI_SWIGLU) ? static_cast<int64_t>(N) : static_cast<int64_t>(2 * N);
  prm.offsets = a->offsets;
  prm.tile_expert = a->tile_expert;
  prm.tile_row = a->tile_row;
  prm.tiles = a->tiles;
  prm.scale = a->scale;
  prm.bias = static_cast<const __nv_bfloat16*>(a->bias);
  prm.scaling = a->scaling;
  prm.out = static_cast<__nv_bfloat16*>(a->out);
  prm.low = static_cast<__nv_bfloat16*>(a->low);
  prm.aux = static_cast<__nv_bfloat16*>(a->aux);
  auto aligned32 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 31u) == 0; };
  prm.a_rows = a->x_rows;
  prm.row_scale = a->row_scale;
  prm.w_grad = a->w_grad;
  prm.w_ld = a->w_ld;
  prm.out_rows = a->out_rows;
  prm.staged = staged;
  if (!staged) tout = tx;  // not read
  if (!staged || epi == MEEP2B_EPI_PLAIN) taux = tx;
  prm.v8 = aligned32(a->out) && (a->aux == nullptr || aligned32(a->aux)) && (a->low == nullptr || aligned32(a->low)) &&
           a->ldo % 16 == 0 && prm.ld_aux % 16 == 0;

  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (a->sm_limit > 0 && a->sm_limit < sms) sms = a->sm_limit;
  const int64_t units = a->max_tiles * prm.nblocks;

  const int block_m = a->block_m == 0 ? 128 : a->block_m;
  if (block_m != 128 && block_m != 256) return MEEP2B_ERR_UNSUPPORTED;
  if (quantised && block_m == 256) return launch_quantized_pair(a, tx, prm, sms, s);
  if (block_m == 256) {
    PairMaps maps;
    maps.x = tx;
    maps.w104 = maps.w96 = maps.w88 = maps.w8 = maps.p16 = maps.u96 = maps.w_mn = maps.p_mn = maps.u_mn = tx;
    maps.out = tout;
    maps.aux = taux;
    if (!a->b_mn) {
      const uint32_t heights[4] = {104, 96, 88, 8};
      CUtensorMap* targets[4] = {&maps.w104, &maps.w96, &maps.w88, &maps.w8};
      for (int i = 0; i < 4; ++i) {
        const uint64_t dims[3] = {K, N, E};
        const uint64_t strides[2] = {K * 2, N * K * 2};
        const uint32_t box[3] = {64, heights[i], 1};
        MEEP2B_TRY(encode_tiled(targets[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a->weight, dims, strides, box,
                                CU_TENSOR_MAP_SWIZZLE_128B));
      }
      if (lora) {
        maps.p16 = tp;
        const uint64_t ud[3] = {RP, N, E};
        const uint64_t us[2] = {RP * 2, N * RP * 2};
        const uint32_t ubx[3] = {RP, 96, 1};
        MEEP2B_TRY(encode_tiled(&maps.u96, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a->up, ud, us, ubx,
                                CU_TENSOR_MAP_SWIZZLE_32B));
      }
    } else {
      if (epi == MEEP2B_EPI_SWIGLU) return MEEP2B_ERR_UNSUPPORTED;
      const uint64_t wd[3] = {N, K, E};
      const uint64_t ws[2] = {N * 2, K * N * 2};
      const uint32_t wb[3] = {32, 64, 1};
      MEEP2B_TRY(encode_tiled(&maps.w_mn, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a->weight, wd, ws, wb,
                              CU_TENSOR_MAP_SWIZZLE_64B));
      if (lora) {
        const uint64_t pd[3] = {RP, K, E};  // the (E, k, 16) panel, 32 columns from column 8 * rank (zeros past 16)
        const uint64_t ps[2] = {RP * 2, K * RP * 2};
        const uint32_t pb[3] = {32, 64, 1};
        MEEP2B_TRY(encode_tiled(&maps.p_mn, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a->panel, pd, ps, pb,
                                CU_TENSOR_MAP_SWIZZLE_64B));
        const uint64_t ud[3] = {N, RP, E};
        const uint64_t us[2] = {N * 2, RP * N * 2};
        const uint32_t ub[3] = {32, RP, 1};
        MEEP2B_TRY(encode_tiled(&maps.u_mn, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a->up, ud, us, ub,
                                CU_TENSOR_MAP_SWIZZLE_64B));
      }
    }
    const int pairs_max = sms / 2;
    const int64_t pairs = units < pairs_max ? (units > 0 ? units : 1) : pairs_max;
    const int grid = static_cast<int>(2 * pairs);
    if (gather) {  // pairs gather the x rows of the K-major SwiGLU product only
      if (a->b_mn || epi != MEEP2B_EPI_SWIGLU) return MEEP2B_ERR_UNSUPPORTED;
      return lora ? launch_pair<false, true, 1, true>(maps, prm, grid, s)
                  : launch_pair<false, false, 1, true>(maps, prm, grid, s);
    }
    if (a->b_mn) {
      if (epi == MEEP2B_EPI_PLAIN)
        return lora ? launch_pair<true, true, 0>(maps, prm, grid, s) : launch_pair<true, false, 0>(maps, prm, grid, s);
      return lora ? launch_pair<true, true, 2>(maps, prm, grid, s) : launch_pair<true, false, 2>(maps, prm, grid, s);
    }
    switch (epi) {
      case MEEP2B_EPI_PLAIN:
        return lora ? launch_pair<false, true, 0>(maps, prm, grid, s) : launch_pair<false, false, 0>(maps, prm, grid, s);
      case MEEP2B_EPI_SWIGLU:
        return lora ? launch_pair<false, true, 1>(maps, prm, grid, s) : launch_pair<false, false, 1>(maps, prm, grid, s);
      default:
        return lora ? launch_pair<false, true, 2>(maps, prm, grid, s) : launch_pair<false, false, 2>(maps, prm, grid, s);
    }
  }
  const int grid = static_cast<int>(units < sms ? (units > 0 ? units : 1) : sms);
  if (quantised) return launch_quantized(a, tx, tp, tu, prm, grid, s);

  const bool mn = a->b_mn != 0;
  if (gather) {
    if (epi == MEEP2B_EPI_SWIGLU)
      return lora ? launch<false, true, 1, true>(tx, tw, tp, tu, tout, taux, prm, grid, s)
                  : launch<false, false, 1, true>(tx, tw, tp, tu, tout, taux, prm, grid, s);
    return lora ? launch<true, true, 2, true>(tx, tw, tp, tu, tout, taux, prm, grid, s)
                : launch<true, false, 2, true>(tx, tw, tp, tu, tout, taux, prm, grid, s);
  }
  switch (epi) {
    case MEEP2B_EPI_PLAIN:
      if (mn) return lora ? launch<true, true, 0>(tx, tw, tp, tu, tout, taux, prm, grid, s) : launch<true, false, 0>(tx, tw, tp, tu, tout, taux, prm, grid, s);
      return lora ? launch<false, true, 0>(tx, tw, tp, tu, tout, taux, prm, grid, s) : launch<false, false, 0>(tx, tw, tp, tu, tout, taux, prm, grid, s);
    case MEEP2B_EPI_SWIGLU:
      return lora ? launch<false, true, 1>(tx, tw, tp, tu, tout, taux, prm, grid, s) : launch<false, false, 1>(tx, tw, tp, tu, tout, taux, prm, grid, s);
    default:
      if (mn) return lora ? launch<true, true, 2>(tx, tw, tp, tu, tout, taux, prm, grid, s) : launch<true, false, 2>(tx, tw, tp, tu, tout, taux, prm, grid, s);
      return lora ? launch<false, true, 2>(tx, tw, tp, tu, tout, taux, prm, grid, s) : launch<false, false, 2>(tx, tw, tp, tu, tout, taux, prm, grid, s);
  }
}

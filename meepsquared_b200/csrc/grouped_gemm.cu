// The grouped product of the expert layer on sm_100a: a persistent, warp-specialised tcgen05 GEMM.
//
// Replaces _grouped_gemm_kernel and _launch (meepsquared/_grouped.py:121-221, 313-345). Rows are sorted by expert;
// a work unit is (tile of 128 rows of one expert, block of 192 output columns). Per CTA (one per SM):
//   warp 0      TMA producer: x tile (128 x 64), the stack tile (192 x 64) with the rank-16 adapter panel P_e
//               riding along as 16 extra rows (K-major) or a 4th column chunk (MN-major), 4-stage ring;
//   warp 1      TMEM owner and MMA issuer: per k-step 4 x tcgen05.mma M=128 N=208 K=16 into one of two
//               accumulators (columns 0..191 the product, 192..207 the panel low = x P_e^T); at the end of the
//               unit two more MMAs of depth 16 add (s low / scale_e) U_e^T into the product, the panel split
//               into hi and lo bf16 planes so that it keeps ~16 bits;
//   warps 4-7   epilogue: TMEM -> registers, scale, bias, (Swi)GLU, bf16, global stores; they also turn the
//               panel into the bf16 operand of that last MMA and store `low` for the backward pass.
// Two accumulators (columns 0 and 256 of a 512-column TMEM allocation) let the epilogue of one unit overlap
// the main loop of the next. Every barrier wait is bounded (common.cuh).
#include "common.cuh"
#include "host.hpp"

namespace meep2b {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int BN = 192;
constexpr int RP = 16;  // rank panel width: the LoRA rank padded to 16
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;    // 16 KB
constexpr int B_BYTES = 4 * 64 * BK * 2;  // 32 KB: room for 4 MN-major chunks (K-major uses 208 rows x 128 B)
constexpr int U_BYTES = BN * RP * 2;    // 6 KB
constexpr int LOW_BYTES = 2 * BM * RP * 2;  // 8 KB: the panel as two bf16 planes, hi and lo
constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
constexpr int OFF_U = OFF_B + STAGES * B_BYTES;
constexpr int OFF_LOW = OFF_U + 2 * U_BYTES;
constexpr int OFF_BAR = OFF_LOW + 2 * LOW_BYTES;
constexpr int NUM_BARS = 2 * STAGES + 13;
constexpr int OFF_TMEM = OFF_BAR + NUM_BARS * 8;
constexpr int SMEM_BYTES = OFF_TMEM + 16 + 1024;  // + slack to align the base to 1024
constexpr int THREADS = 256;
constexpr uint32_t TMEM_COLS = 512;
constexpr int ACC_STRIDE = 256;

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
};

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

template <bool B_MN, bool LORA, int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                        const __grid_constant__ CUtensorMap tm_p, const __grid_constant__ CUtensorMap tm_u,
                        const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const uint32_t bar0 = sbase + OFF_BAR;
  auto bar_full = [&](int s) { return bar0 + 8u * s; };
  auto bar_empty = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto bar_tfull = [&](int b) { return bar0 + 8u * (2 * STAGES + b); };
  auto bar_tempty = [&](int b) { return bar0 + 8u * (2 * STAGES + 2 + b); };
  auto bar_lowfull = [&](int b) { return bar0 + 8u * (2 * STAGES + 4 + b); };
  auto bar_lowready = [&](int b) { return bar0 + 8u * (2 * STAGES + 6 + b); };
  auto bar_ufull = [&](int b) { return bar0 + 8u * (2 * STAGES + 8 + b); };
  auto bar_uempty = [&](int b) { return bar0 + 8u * (2 * STAGES + 10 + b); };
  const uint32_t bar_drain = bar0 + 8u * (2 * STAGES + 12);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_TMEM);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full(s), 1);
      mbar_init(bar_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_tfull(b), 1);
      mbar_init(bar_tempty(b), 128);
      mbar_init(bar_lowfull(b), 1);
      mbar_init(bar_lowready(b), 128);
      mbar_init(bar_ufull(b), 1);
      mbar_init(bar_uempty(b), 1);
    }
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
  constexpr int NW = BN;  // output columns per unit (SwiGLU: 96 gate + 96 up)

  if (warp == 0) {
    // ------------------------------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_w);
      if (LORA) {
        tma_prefetch_desc(&tm_p);
        tma_prefetch_desc(&tm_u);
      }
      constexpr uint32_t B_TX = 64 * NW * 2 + (LORA ? (B_MN ? 64 * 64 * 2 : RP * 64 * 2) : 0);
      constexpr uint32_t STAGE_TX = A_BYTES + B_TX;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t last_parity[STAGES];
      bool issued[STAGES];
      for (int s = 0; s < STAGES; ++s) issued[s] = false, last_parity[s] = 0;
      bool ok = true;
      int it = 0;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ++it) {
        const int t = u / p.nblocks, nb = u - t * p.nblocks;
        const int e = p.tile_expert[t], row0 = p.tile_row[t];
        if (LORA) {
          const int ub = it & 1;
          const uint32_t uph = (it >> 1) & 1;
          if (!mbar_wait(bar_uempty(ub), uph ^ 1)) { ok = false; break; }
          const uint32_t dst = sbase + OFF_U + ub * U_BYTES;
          mbar_arrive_expect_tx(bar_ufull(ub), U_BYTES);
          if (!B_MN) {
            if (EPI == MEEP2B_EPI_SWIGLU) {
              tma_load_3d(dst, &tm_u, bar_ufull(ub), 0, nb * 96, e);
              tma_load_3d(dst + 96 * RP * 2, &tm_u, bar_ufull(ub), 0, p.inter + nb * 96, e);
            } else {
              tma_load_3d(dst, &tm_u, bar_ufull(ub), 0, nb * BN, e);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 3; ++j) tma_load_3d(dst + j * 2048, &tm_u, bar_ufull(ub), nb * BN + 64 * j, 0, e);
          }
        }
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait(bar_empty(stage), phase ^ 1)) { ok = false; break; }
          const uint32_t fb = bar_full(stage);
          const uint32_t a_dst = sbase + OFF_A + stage * A_BYTES;
          const uint32_t b_dst = sbase + OFF_B + stage * B_BYTES;
          mbar_arrive_expect_tx(fb, STAGE_TX);
          tma_load_2d(a_dst, &tm_x, fb, kb * BK, row0);
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
          issued[stage] = true;
          last_parity[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // a partner is gone: let this thread's copies in flight land before the CTA's shared memory goes away
        for (int s = 0; s < STAGES; ++s)
          if (issued[s]) mbar_wait_drain(bar_full(s), last_parity[s]);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_MAIN = idesc_bf16(BM, LORA ? BN + RP : BN, false, B_MN);
      constexpr uint32_t IDESC_UP = idesc_bf16(BM, BN, false, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ++it) {
        const int ab = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        if (!mbar_wait(bar_tempty(ab), aph ^ 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem_base + ab * ACC_STRIDE;
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait(bar_full(stage), phase)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = sbase + OFF_A + stage * A_BYTES;
          const uint32_t b_addr = sbase + OFF_B + stage * B_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t adesc = smem_desc(a_addr + kk * 32, 16, 1024, 2);
            const uint64_t bdesc =
                B_MN ? smem_desc(b_addr + kk * 2048, 8192, 1024, 2) : smem_desc(b_addr + kk * 32, 16, 1024, 2);
            mma_bf16(d, adesc, bdesc, IDESC_MAIN, (kb | kk) != 0);
          }
          mma_commit(bar_empty(stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if (LORA) {
          mma_commit(bar_lowfull(ab));
          if (!mbar_wait(bar_lowready(ab), aph)) { ok = false; break; }
          if (!mbar_wait(bar_ufull(ab), aph)) { ok = false; break; }
          tc_fence_after();
          const uint32_t low_addr = sbase + OFF_LOW + ab * LOW_BYTES;
          const uint32_t u_addr = sbase + OFF_U + ab * U_BYTES;
          const uint64_t bdesc = B_MN ? smem_desc(u_addr, 2048, 1024, 2) : smem_desc(u_addr, 16, 256, 6);
          mma_bf16(d, smem_desc(low_addr, 16, 256, 6), bdesc, IDESC_UP, 1);             // hi plane
          mma_bf16(d, smem_desc(low_addr + BM * RP * 2, 16, 256, 6), bdesc, IDESC_UP, 1);  // lo plane
          mma_commit(bar_uempty(ab));
        }
        mma_commit(bar_tfull(ab));
      }
      if (!ok) {
        // let the MMAs already issued finish before tensor memory is released
        mma_commit(bar_drain);
        mbar_wait_drain(bar_drain, 0);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int r_in = q * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    int it = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x, ++it) {
      const int t = u / p.nblocks, nb = u - t * p.nblocks;
      const int e = p.tile_expert[t];
      const int row = p.tile_row[t] + r_in;
      const bool valid = row < p.offsets[e];
      const int ab = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      const float sc = p.scale != nullptr ? p.scale[e] : 1.0f;
      const uint32_t d = tmem_base + lane_base + ab * ACC_STRIDE;
      if (LORA) {
        if (!mbar_wait(bar_lowfull(ab), aph)) break;
        tc_fence_after();
        float lv[16];
        tmem_ld16(d + BN, lv);
        uint32_t lw[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) lw[i] = pack_bf16x2(lv[2 * i], lv[2 * i + 1]);
        if (p.low != nullptr && nb == 0 && valid) {
          uint4* dst = reinterpret_cast<uint4*>(p.low + static_cast<int64_t>(row) * RP);
          dst[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
          dst[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
        }
        // the A operand of the last MMAs: a = s * low / scale_e (float32) split into two bf16 planes, hi = bf16(a)
        // and lo = bf16(a - hi), so the adapter's second product keeps ~16 bits of the panel, not 8.
        // K-major with the 32-byte swizzle.
        const float f = p.scaling / sc;
        uint32_t hw[8], lo_w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float a0 = lv[2 * i] * f, a1 = lv[2 * i + 1] * f;
          hw[i] = pack_bf16x2(a0, a1);
          lo_w[i] = pack_bf16x2(a0 - bf16_lo(hw[i]), a1 - bf16_hi(hw[i]));
        }
        uint8_t* low_row = smem + OFF_LOW + ab * LOW_BYTES + r_in * 32;
        const int sw = (r_in >> 2) & 1;
        *reinterpret_cast<uint4*>(low_row + (0 ^ sw) * 16) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(low_row + (1 ^ sw) * 16) = make_uint4(hw[4], hw[5], hw[6], hw[7]);
        uint8_t* lo_row = low_row + BM * RP * 2;
        *reinterpret_cast<uint4*>(lo_row + (0 ^ sw) * 16) = make_uint4(lo_w[0], lo_w[1], lo_w[2], lo_w[3]);
        *reinterpret_cast<uint4*>(lo_row + (1 ^ sw) * 16) = make_uint4(lo_w[4], lo_w[5], lo_w[6], lo_w[7]);
        fence_proxy_async_smem();
        mbar_arrive(bar_lowready(ab));
      }
      if (!mbar_wait(bar_tfull(ab), aph)) break;
      tc_fence_after();
      const int64_t orow = static_cast<int64_t>(row);
      if (EPI == MEEP2B_EPI_PLAIN) {
        const int n0 = nb * BN;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          const int col = n0 + 32 * c;
          if (col >= p.N) break;
          float v[32];
          tmem_ld32(d + 32 * c, v);
          if (valid) {
            const __nv_bfloat16* bias = p.bias != nullptr ? p.bias + static_cast<int64_t>(e) * p.N + col : nullptr;
            __nv_bfloat16* dst = p.out + orow * p.ldo + col;
            if (col + 32 <= p.N) {
              uint32_t w[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                float a = v[2 * j] * sc, b = v[2 * j + 1] * sc;
                if (bias != nullptr) {
                  a += __bfloat162float(bias[2 * j]);
                  b += __bfloat162float(bias[2 * j + 1]);
                }
                w[j] = pack_bf16x2(a, b);
              }
              uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
              for (int j = 0; j < 4; ++j) d4[j] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
            } else {
              for (int j = 0; j < p.N - col; ++j) {
                float a = v[j] * sc;
                if (bias != nullptr) a += __bfloat162float(bias[j]);
                dst[j] = __float2bfloat16_rn(a);
              }
            }
          }
        }
      } else if (EPI == MEEP2B_EPI_SWIGLU) {
        const int n0h = nb * 96;
#pragma unroll 1
        for (int c = 0; c < 3; ++c) {
          const int col = n0h + 32 * c;
          if (col >= p.inter) break;
          float g[32], uu[32];
          tmem_ld32(d + 32 * c, g);
          tmem_ld32(d + 96 + 32 * c, uu);
          if (valid) {
            const int cnt = min(32, p.inter - col);
            const __nv_bfloat16* bias_g =
                p.bias != nullptr ? p.bias + static_cast<int64_t>(e) * p.N + col : nullptr;
            __nv_bfloat16* pre = p.aux + orow * p.ld_aux;
            __nv_bfloat16* h = p.out + orow * p.ldo + col;
            uint32_t gw[16], uw[16], hw[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              float g0 = g[2 * j] * sc, g1 = g[2 * j + 1] * sc;
              float u0 = uu[2 * j] * sc, u1 = uu[2 * j + 1] * sc;
              if (bias_g != nullptr && 2 * j + 1 < cnt) {
                g0 += __bfloat162float(bias_g[2 * j]);
                g1 += __bfloat162float(bias_g[2 * j + 1]);
                u0 += __bfloat162float(bias_g[p.inter + 2 * j]);
                u1 += __bfloat162float(bias_g[p.inter + 2 * j + 1]);
              }
              gw[j] = pack_bf16x2(g0, g1);
              uw[j] = pack_bf16x2(u0, u1);
              const float a0 = bf16_round(silu_f(bf16_lo(gw[j]))), a1 = bf16_round(silu_f(bf16_hi(gw[j])));
              hw[j] = pack_bf16x2(a0 * bf16_lo(uw[j]), a1 * bf16_hi(uw[j]));
            }
            if (cnt == 32) {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                reinterpret_cast<uint4*>(pre + col)[j] = make_uint4(gw[4 * j], gw[4 * j + 1], gw[4 * j + 2], gw[4 * j + 3]);
                reinterpret_cast<uint4*>(pre + p.inter + col)[j] =
                    make_uint4(uw[4 * j], uw[4 * j + 1], uw[4 * j + 2], uw[4 * j + 3]);
                reinterpret_cast<uint4*>(h)[j] = make_uint4(hw[4 * j], hw[4 * j + 1], hw[4 * j + 2], hw[4 * j + 3]);
              }
            } else {
              for (int j = 0; j < cnt; ++j) {
                const uint32_t sh = (j & 1) * 16;
                pre[col + j] = __ushort_as_bfloat16(static_cast<unsigned short>(gw[j >> 1] >> sh));
                pre[p.inter + col + j] = __ushort_as_bfloat16(static_cast<unsigned short>(uw[j >> 1] >> sh));
                h[j] = __ushort_as_bfloat16(static_cast<unsigned short>(hw[j >> 1] >> sh));
              }
            }
          }
        }
      } else {  // MEEP2B_EPI_DSWIGLU: the product is dh; aux holds (gate, up); out receives (dgate, dup)
        const int n0 = nb * BN;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          const int col = n0 + 32 * c;
          if (col >= p.N) break;
          float v[32];
          tmem_ld32(d + 32 * c, v);
          if (valid) {
            const int cnt = min(32, p.N - col);
            const __nv_bfloat16* gp = p.aux + orow * p.ld_aux + col;
            const __nv_bfloat16* up = gp + p.N;
            __nv_bfloat16* dg = p.out + orow * p.ldo + col;
            __nv_bfloat16* du = dg + p.N;
            uint32_t gw[16], uw[16], dgw[16], duw[16];
            if (cnt == 32) {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const uint4 a = reinterpret_cast<const uint4*>(gp)[j], b = reinterpret_cast<const uint4*>(up)[j];
                gw[4 * j] = a.x, gw[4 * j + 1] = a.y, gw[4 * j + 2] = a.z, gw[4 * j + 3] = a.w;
                uw[4 * j] = b.x, uw[4 * j + 1] = b.y, uw[4 * j + 2] = b.z, uw[4 * j + 3] = b.w;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const uint32_t g0 = 2 * j < cnt ? __bfloat16_as_ushort(gp[2 * j]) : 0u;
                const uint32_t g1 = 2 * j + 1 < cnt ? __bfloat16_as_ushort(gp[2 * j + 1]) : 0u;
                const uint32_t u0 = 2 * j < cnt ? __bfloat16_as_ushort(up[2 * j]) : 0u;
                const uint32_t u1 = 2 * j + 1 < cnt ? __bfloat16_as_ushort(up[2 * j + 1]) : 0u;
                gw[j] = g0 | (g1 << 16);
                uw[j] = u0 | (u1 << 16);
              }
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              float dgo[2], duo[2];
#pragma unroll
              for (int hlf = 0; hlf < 2; ++hlf) {
                const float gb = hlf ? bf16_hi(gw[j]) : bf16_lo(gw[j]);
                const float ub = hlf ? bf16_hi(uw[j]) : bf16_lo(uw[j]);
                const float dh = bf16_round(v[2 * j + hlf] * sc);
                const float sig = 1.0f / (1.0f + expf(-gb));
                const float act = bf16_round(silu_f(gb));
                const float dact = bf16_round(dh * ub);
                duo[hlf] = dh * act;
                dgo[hlf] = dact * sig * (1.0f + gb * (1.0f - sig));
              }
              dgw[j] = pack_bf16x2(dgo[0], dgo[1]);
              duw[j] = pack_bf16x2(duo[0], duo[1]);
            }
            if (cnt == 32) {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                reinterpret_cast<uint4*>(dg)[j] = make_uint4(dgw[4 * j], dgw[4 * j + 1], dgw[4 * j + 2], dgw[4 * j + 3]);
                reinterpret_cast<uint4*>(du)[j] = make_uint4(duw[4 * j], duw[4 * j + 1], duw[4 * j + 2], duw[4 * j + 3]);
              }
            } else {
              for (int j = 0; j < cnt; ++j) {
                const uint32_t sh = (j & 1) * 16;
                dg[j] = __ushort_as_bfloat16(static_cast<unsigned short>(dgw[j >> 1] >> sh));
                du[j] = __ushort_as_bfloat16(static_cast<unsigned short>(duw[j >> 1] >> sh));
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(bar_tempty(ab));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <bool B_MN, bool LORA, int EPI>
static int launch(const CUtensorMap& tx, const CUtensorMap& tw, const CUtensorMap& tp, const CUtensorMap& tu,
                  const Params& prm, int grid, cudaStream_t s) {
  auto kern = grouped_gemm_kernel<B_MN, LORA, EPI>;
  static bool configured = false;  // per instantiation; attributes are per device but idempotent
  if (!configured) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess) {
      cudaGetLastError();
      return MEEP2B_ERR_LAUNCH;
    }
    configured = true;
  }
  kern<<<grid, THREADS, SMEM_BYTES, s>>>(tx, tw, tp, tu, prm);
  return launch_status();
}

}  // namespace gemm
}  // namespace meep2b

using namespace meep2b;
using namespace meep2b::gemm;

extern "C" int meep2b_grouped_product(const meep2b_product* a, void* stream) {
  if (a == nullptr) return MEEP2B_ERR_SHAPE;
  if (a->weight_dtype != MEEP2B_BF16) return MEEP2B_ERR_UNSUPPORTED;
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
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  if (a->rows == 0) return MEEP2B_OK;

  const uint64_t K = a->k, N = a->n, E = a->experts, rows = a->rows;
  CUtensorMap tx, tw, tp, tu;
  {
    const uint64_t dims[2] = {K, rows};
    const uint64_t strides[1] = {static_cast<uint64_t>(a->ldx) * 2};
    const uint32_t box[2] = {64, 128};
    MEEP2B_TRY(encode_tiled(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a->x, dims, strides, box,
                            CU_TENSOR_MAP_SWIZZLE_128B));
  }
  const uint32_t rows_per_load = (epi == MEEP2B_EPI_SWIGLU) ? 96 : BN;
  if (!a->b_mn) {
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
      const uint64_t pd[3] = {64, K, E};
      const uint64_t ps[2] = {128, K * 128};
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

  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (a->sm_limit > 0 && a->sm_limit < sms) sms = a->sm_limit;
  const int64_t units = a->max_tiles * prm.nblocks;
  const int grid = static_cast<int>(units < sms ? (units > 0 ? units : 1) : sms);

  const bool mn = a->b_mn != 0;
  switch (epi) {
    case MEEP2B_EPI_PLAIN:
      if (mn) return lora ? launch<true, true, 0>(tx, tw, tp, tu, prm, grid, s) : launch<true, false, 0>(tx, tw, tp, tu, prm, grid, s);
      return lora ? launch<false, true, 0>(tx, tw, tp, tu, prm, grid, s) : launch<false, false, 0>(tx, tw, tp, tu, prm, grid, s);
    case MEEP2B_EPI_SWIGLU:
      return lora ? launch<false, true, 1>(tx, tw, tp, tu, prm, grid, s) : launch<false, false, 1>(tx, tw, tp, tu, prm, grid, s);
    default:
      if (mn) return lora ? launch<true, true, 2>(tx, tw, tp, tu, prm, grid, s) : launch<true, false, 2>(tx, tw, tp, tu, prm, grid, s);
      return lora ? launch<false, true, 2>(tx, tw, tp, tu, prm, grid, s) : launch<false, false, 2>(tx, tw, tp, tu, prm, grid, s);
  }
}

// The grouped product with a quantised stack, dequantised in shared memory between the TMA load and the MMA.
//
// Included by grouped_gemm.cu inside namespace meep2b::gemm (it shares the tile geometry, Params and the epilogue).
// Weight formats (the reference's dequantisations, restated per element in the converter), each 64 consecutive
// weights of a stored row sharing one float32 multiplier m (TMA-loaded beside the codes, prepared once per frozen
// stack by meep2b_quant_multipliers as (experts, cols/64, rows)):
//   NF4          w = bf16(NF4[code] * m), m the block's absmax_f32 (bitsandbytes' cdequantize_blockwise_bf16_nf4,
//                called by meepsquared/_vendor/axolotl/quantize.py:85-96)
//   E4M3         w = bf16(e4m3) exactly, the per-expert scale applied to the accumulator in the epilogue
//                (meepsquared/_grouped.py:200-201 converts the FP8 tile to bf16 and :207-208 scales the result)
//   E4M3_BLOCKS  w = bf16(bf16(e4m3) * m), m = bf16(scale) of the block (quantize.py:131-157 dequantize_fp8)
// so the MMA sees exactly the bf16 stack the reference's dequantisation gives, and the product equals the one
// over a stack dequantised beforehand, bit for bit. The e4m3 codes become bf16 with integer operations and one
// bf16x2 multiply by 2^120 (the code's bits placed in a bf16 with the exponent field shifted; exact, subnormal
// codes included), not with the float conversion instructions, whose throughput is a fraction of the ALU's.
//
// Per CTA (one per SM), 16 warps:
//   warp 0       TMA producer: per k-step the x tile, the LoRA panel (bf16) and the raw quantised B tile (codes,
//                swizzled) into ring 1; the deferred up factor as in the bf16 kernel;
//   warp 1       TMEM owner and MMA issuer: A from ring 1, B from ring 2;
//   warps 2-11   converters (320 threads, a few 8-weight tasks each per k-step): raw codes of ring 1 -> bf16 B
//                tile of ring 2 in the 128-byte-swizzled layout the MMA reads (what TMA writes for a bf16 stack),
//                plus a copy of the panel rows;
//   warps 12-15  epilogue, one warp per TMEM lane quarter taking both column halves of a unit in turn
// (dSwiGLU products: warps 2-7 convert and warps 8-15 run the epilogue, as QRoles says).
// Registers: launched with 128 per thread (512 threads); the roles' warpgroups give theirs down with setmaxnreg and
// the epilogue's take 176, to the launch's total of 65536.

enum QuantFormat { QF_NF4 = 1, QF_E4M3 = 2, QF_E4M3_BLOCKS = 3 };

constexpr int Q_THREADS = 512;
constexpr int Q_CONV_WARP0 = 2;

// Converter warps per CTA: ten (warps 2-11), with one epilogue warp per TMEM lane quarter (warps 12-15) taking both
// column halves of a unit in turn; six (warps 2-7) for the dSwiGLU products over e4m3 codes, whose epilogue (the
// pre-activations read back and the SwiGLU derivative per element) then bounds the unit and needs two warps per
// lane quarter (warps 8-15, one half each). NF4's conversion (a level look-up per weight) keeps ten converters
// throughout (measured faster). Registers: 3 x 128 x 112 + 128 x 176, or 2 x 128 x 80 + 2 x 128 x 176
// (setmaxnreg), 65536 either way.
template <int EPI, int QF>
struct QRoles {
  static constexpr int CONV_WARPS = EPI == MEEP2B_EPI_DSWIGLU && QF != QF_NF4 ? 6 : 10;
  static constexpr int CONV_THREADS = CONV_WARPS * 32;
  static constexpr int EPI_WARP0 = Q_CONV_WARP0 + CONV_WARPS;
  static constexpr int EPI_HALVES = EPI_WARP0 == 8 ? 1 : 2;  // column halves each epilogue warp takes
};

// Shared memory: ring 1 (S1 stages) = x tile | panel | raw codes | multipliers; ring 2 (S2 stages) = bf16 B tile
// (+ panel rows).
template <bool B_MN, int QF>
struct QPlan {
  static constexpr int PANEL_BYTES = B_MN ? 64 * BK * 2 : RP * BK * 2;  // one 64-column chunk : 16 rows
  // raw codes: rows of one 64-weight group (32 bytes NF4, 64 bytes e4m3), swizzled by TMA (32- or 64-byte pattern)
  // so that converter threads reading consecutive rows hit distinct banks. K-major: 192 rows; MN-major: three
  // regions (one per 64-column group) of 64 k rows.
  static constexpr int RAW_ROW = QF == QF_NF4 ? 32 : 64;
  static constexpr int RAW_ROWS = B_MN ? 3 * BK : BN;
  static constexpr int RAW_BYTES = RAW_ROW * RAW_ROWS;
  static constexpr int MULT_BYTES = QF == QF_E4M3 ? 0 : 1024;  // 192 floats (K-major rows; MN: 3 groups x 64)
  static constexpr int MULT_TX = QF == QF_E4M3 ? 0 : 192 * 4;
  static constexpr int OFF_RAW = A_BYTES + PANEL_BYTES;
  static constexpr int OFF_MULT = OFF_RAW + RAW_BYTES;
  static constexpr int S1_BYTES = A_BYTES + PANEL_BYTES + RAW_BYTES + MULT_BYTES;
  static constexpr int B_BYTES = B_MN ? 4 * 64 * BK * 2 : (BN + RP) * BK * 2;
  static constexpr int S2 = B_MN ? 2 : 3;
  static constexpr int BUDGET = 232448 - 1024 - 1024 - 512;  // less alignment slack, the NF4 levels, barriers
  static constexpr int S1_FIT = (BUDGET - S2 * B_BYTES - U_BYTES - LOW_BYTES) / S1_BYTES;
  static constexpr int S1 = S1_FIT > 5 ? 5 : S1_FIT;
  static constexpr int OFF_R1 = 0;
  static constexpr int OFF_R2 = OFF_R1 + S1 * S1_BYTES;
  static constexpr int OFF_U = OFF_R2 + S2 * B_BYTES;
  static constexpr int OFF_LOW = OFF_U + U_BYTES;
  static constexpr int OFF_LUT = OFF_LOW + LOW_BYTES;
  static constexpr int OFF_BAR = OFF_LUT + 1024;
  static constexpr int NUM_BARS = 2 * S1 + 2 * S2 + 10;
  static constexpr int OFF_TMEM = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_TMEM + 16 + 1024;
  static_assert(S1 >= 3, "the quantised ring needs three stages");
  static_assert(SMEM_BYTES <= 232448, "quantised plan exceeds 227 KB");
  static_assert(S1_BYTES % 1024 == 0 && B_BYTES % 1024 == 0 && OFF_U % 1024 == 0 && OFF_LOW % 1024 == 0,
                "swizzled tiles need 1 KB alignment");
};



// Shared-memory accesses by shared-window address (ld/st.shared: no generic-address resolution on the path).
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds_v2(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ float lds_f32(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ void sts_v4(uint32_t a, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

// 8 bf16 from 4 code bytes of NF4 (two codes a byte, the first in the high nibble), each bf16(level * m): the 16
// levels are read from shared memory at lv (one word per level: a warp's reads hit distinct banks or broadcast).
__device__ __forceinline__ uint4 nf4_chunk(uint32_t w, float m, uint32_t lv) {
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t b = (w >> (8 * j)) & 0xFFu;
    o[j] = pack_bf16x2(__fmul_rn(lds_f32(lv + 4u * (b >> 4)), m), __fmul_rn(lds_f32(lv + 4u * (b & 15u)), m));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// 8 bf16 from 8 e4m3 codes: exactly (E4M3), or times the bf16 multiplier m2 and rounded once (E4M3_BLOCKS: the
// product of a 4-bit and an 8-bit significand is exact in float32, so the bf16 multiply rounds as
// bf16(float32(w8) * bf16(s)) does).
template <int QF>
__device__ __forceinline__ uint4 e4m3_chunk(uint2 c, __nv_bfloat162 m2) {
  uint32_t o[4];
  const uint32_t words[2] = {c.x, c.y};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __nv_bfloat162 v = e4m3x2_to_bf16x2(words[j >> 1], (j & 1) ? 0x3424u : 0x1404u);
    if (QF == QF_E4M3_BLOCKS) v = __hmul2(v, m2);
    o[j] = *reinterpret_cast<uint32_t*>(&v);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// The converters' share of a k-step: the raw codes of `rows` B rows into the bf16 B tile, in tasks of 8 weights.
// Task q is chunk c = q % 8 of B row r = q / 8: its 8 weights become one 16-byte chunk of the row's 128 bytes, so
// the eight chunks of a row go to eight consecutive threads, which read the row's codes as one 64-byte (e4m3) or
// 32-byte (NF4) run and write its bf16 chunks as one 128-byte row (no bank conflicts either way). Both B layouts
// put row r (K-major: a stored row; MN-major: 64-column group r / 64, k row r % 64) at byte r * 128 with the chunk
// swizzle r % 8, its codes at raw row r (16-byte chunk j at j ^ (r / 4 % 2) for NF4's 32-byte swizzle, j ^ (r / 2
// % 4) for e4m3's 64-byte one) and its multiplier at mult[r]. A thread's code loads are all issued before its
// conversions; rows for which valid(r) is false (past the stack's end) are written as zeros.
template <int QF, int ROWS, int NT, typename Valid>
__device__ __forceinline__ void convert_tasks(int ct, int rows, const uint8_t* raw, const float* mult, uint8_t* bdst,
                                              const float* lv, Valid valid) {
  constexpr int RAW_ROW = QF == QF_NF4 ? 32 : 64;
  constexpr int MAXT = (ROWS * 8 + NT - 1) / NT;
  const int total = rows * 8;
  const uint32_t raw_s = smem_u32(raw), mult_s = smem_u32(mult), bdst_s = smem_u32(bdst), lv_s = smem_u32(lv);
  uint2 code[MAXT];
  float m[MAXT];
#pragma unroll
  for (int i = 0; i < MAXT; ++i) {
    const int q = ct + i * NT;
    code[i] = make_uint2(0u, 0u);
    m[i] = 1.0f;
    if (q < total) {
      const int r = q >> 3, c = q & 7;
      const uint32_t src = raw_s + static_cast<uint32_t>(r * RAW_ROW);
      if (QF == QF_NF4) {
        const uint32_t rsw = (r >> 2) & 1;
        code[i].x = lds_u32(src + (((static_cast<uint32_t>(c) >> 2) ^ rsw) << 4) + ((c & 3) << 2));
      } else {
        const uint32_t rsw = (r >> 1) & 3;
        code[i] = lds_v2(src + (((static_cast<uint32_t>(c) >> 1) ^ rsw) << 4) + ((c & 1) << 3));
      }
      if (QF != QF_E4M3) m[i] = lds_f32(mult_s + 4u * static_cast<uint32_t>(r));
    }
  }
#pragma unroll
  for (int i = 0; i < MAXT; ++i) {
    const int q = ct + i * NT;
    if (q < total) {
      const int r = q >> 3, c = q & 7;
      uint4 o;
      if (!valid(r)) {
        o = make_uint4(0u, 0u, 0u, 0u);
      } else if (QF == QF_NF4) {
        o = nf4_chunk(code[i].x, m[i], lv_s);
      } else {
        o = e4m3_chunk<QF>(code[i], __float2bfloat162_rn(m[i]));  // m holds a bf16 value: exact
      }
      sts_v4(bdst_s + static_cast<uint32_t>(r * 128) + ((static_cast<uint32_t>(c) ^ static_cast<uint32_t>(r & 7)) << 4),
             o);
    }
  }
}

// Warps 0-7 of the quantised kernel: TMA producer, MMA issuer, converters.
template <bool B_MN, bool LORA, int EPI, int QF>
__device__ __forceinline__ void q_mainloop_roles(const CUtensorMap& tm_x, const CUtensorMap& tm_raw,
                                                 const CUtensorMap& tm_mult, const CUtensorMap& tm_p,
                                                 const CUtensorMap& tm_u, const Params& p, uint8_t* smem,
                                                 uint32_t sbase, uint32_t tmem_base, int total, int warp, int lane) {
  using QP = QPlan<B_MN, QF>;
  constexpr int S1 = QP::S1, S2 = QP::S2;
  constexpr bool SWIGLU = EPI == MEEP2B_EPI_SWIGLU;
  const uint32_t bar0 = sbase + QP::OFF_BAR;
  auto bar_full1 = [&](int s) { return bar0 + 8u * s; };
  auto bar_empty1 = [&](int s) { return bar0 + 8u * (S1 + s); };
  auto bar_full2 = [&](int s) { return bar0 + 8u * (2 * S1 + s); };
  auto bar_empty2 = [&](int s) { return bar0 + 8u * (2 * S1 + S2 + s); };
  const uint32_t bar1 = bar0 + 8u * (2 * S1 + 2 * S2);
  auto bar_tfull = [&](int b) { return bar1 + 8u * b; };
  auto bar_tempty = [&](int b) { return bar1 + 8u * (2 + b); };
  auto bar_lowfull = [&](int b) { return bar1 + 8u * (4 + b); };
  const uint32_t bar_lowready = bar1 + 8u * 6;
  const uint32_t bar_ufull = bar1 + 8u * 7;
  const uint32_t bar_uempty = bar1 + 8u * 8;
  const uint32_t bar_drain = bar1 + 8u * 9;
  const float* lv = reinterpret_cast<const float*>(smem + QP::OFF_LUT);

  if (warp == 0) {
    // ------------------------------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_raw);
      if (QF != QF_E4M3) tma_prefetch_desc(&tm_mult);
      if (LORA) {
        tma_prefetch_desc(&tm_p);
        tma_prefetch_desc(&tm_u);
      }
      constexpr uint32_t STAGE_TX = A_BYTES + (LORA ? QP::PANEL_BYTES : 0) + QP::RAW_BYTES + QP::MULT_TX;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t last_parity[S1];
      bool issued[S1];
      for (int s = 0; s < S1; ++s) issued[s] = false, last_parity[s] = 0;
      bool ok = true;
      int it = 0;
      int pu = -1, pu_nb = 0, pu_e = 0;  // the up factor goes out one k-step into the next unit
      auto load_u = [&]() -> bool {
        if (!mbar_wait(bar_uempty, (pu & 1) ^ 1)) return false;
        const uint32_t dst = sbase + QP::OFF_U;
        mbar_arrive_expect_tx(bar_ufull, U_BYTES);
        if (!B_MN) {
          if (SWIGLU) {
            tma_load_3d(dst, &tm_u, bar_ufull, 0, pu_nb * 96, pu_e);
            tma_load_3d(dst + 96 * RP * 2, &tm_u, bar_ufull, 0, p.inter + pu_nb * 96, pu_e);
          } else {
            tma_load_3d(dst, &tm_u, bar_ufull, 0, pu_nb * BN, pu_e);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 3; ++j) tma_load_3d(dst + j * 2048, &tm_u, bar_ufull, pu_nb * BN + 64 * j, 0, pu_e);
        }
        pu = -1;
        return true;
      };
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ++it) {
        const int t = u / p.nblocks, nb = u - t * p.nblocks;
        const int e = p.tile_expert[t], row0 = p.tile_row[t];
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait(bar_empty1(stage), phase ^ 1)) { ok = false; break; }
          const uint32_t fb = bar_full1(stage);
          const uint32_t s_dst = sbase + QP::OFF_R1 + stage * QP::S1_BYTES;
          const uint32_t r_dst = s_dst + QP::OFF_RAW;
          const uint32_t m_dst = s_dst + QP::OFF_MULT;
          mbar_arrive_expect_tx(fb, STAGE_TX);
          tma_load_2d(s_dst, &tm_x, fb, kb * BK, row0);
          if (LORA) {
            if (!B_MN) tma_load_3d(s_dst + A_BYTES, &tm_p, fb, kb * BK, 0, e);
            else tma_load_3d(s_dst + A_BYTES, &tm_p, fb, 0, kb * BK, e);
          }
          constexpr int BPE = QF == QF_NF4 ? 1 : 2;  // code bytes are (elements * BPE) / 2
          // the multipliers: (experts, cols/64, rows) float32, x = the stored row, y = the 64-column group
          if (!B_MN) {
            if (SWIGLU) {
              tma_load_3d(r_dst, &tm_raw, fb, kb * BK * BPE / 2, nb * 96, e);
              tma_load_3d(r_dst + 96 * QP::RAW_ROW, &tm_raw, fb, kb * BK * BPE / 2, p.inter + nb * 96, e);
              if (QF != QF_E4M3) {
                tma_load_3d(m_dst, &tm_mult, fb, nb * 96, kb, e);
                tma_load_3d(m_dst + 96 * 4, &tm_mult, fb, p.inter + nb * 96, kb, e);
              }
            } else {
              tma_load_3d(r_dst, &tm_raw, fb, kb * BK * BPE / 2, nb * BN, e);
              if (QF != QF_E4M3) tma_load_3d(m_dst, &tm_mult, fb, nb * BN, kb, e);
            }
          } else {
#pragma unroll
            for (int g = 0; g < 3; ++g)
              tma_load_3d(r_dst + g * BK * QP::RAW_ROW, &tm_raw, fb, (nb * BN + 64 * g) * BPE / 2, kb * BK, e);
            if (QF != QF_E4M3) tma_load_3d(m_dst, &tm_mult, fb, kb * BK, nb * 3, e);
          }
          issued[stage] = true;
          last_parity[stage] = phase;
          if (++stage == S1) {
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
      if (!ok) {
        for (int s = 0; s < S1; ++s)
          if (issued[s]) mbar_wait_drain(bar_full1(s), last_parity[s]);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_MAIN = idesc_bf16(BM, LORA ? BN + RP : BN, false, B_MN);
      constexpr uint32_t IDESC_UP = idesc_bf16(BM, BN, false, B_MN);
      int s1 = 0, s2 = 0;
      uint32_t ph1 = 0, ph2 = 0;
      bool ok = true;
      int it = 0;
      int pend = -1;
      auto issue_up = [&](bool block) -> bool {
        const uint32_t par = static_cast<uint32_t>(pend) & 1;
        if (block) {
          if (!mbar_wait(bar_lowready, par) || !mbar_wait(bar_ufull, par)) return false;
        } else if (!mbar_test(bar_lowready, par) || !mbar_test(bar_ufull, par)) {
          return true;
        }
        tc_fence_after();
        const uint32_t dp = tmem_base + (pend & 1) * ACC_STRIDE;
        const uint32_t low_addr = sbase + QP::OFF_LOW;
        const uint32_t u_addr = sbase + QP::OFF_U;
        const uint64_t bdesc = B_MN ? smem_desc(u_addr, 2048, 1024, 2) : smem_desc(u_addr, 16, 256, 6);
        mma_bf16(dp, smem_desc(low_addr, 16, 256, 6), bdesc, IDESC_UP, 1);
        mma_bf16(dp, smem_desc(low_addr + BM * RP * 2, 16, 256, 6), bdesc, IDESC_UP, 1);
        mma_commit(bar_uempty);
        mma_commit(bar_tfull(pend & 1));
        pend = -1;
        return true;
      };
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ++it) {
        const int ab = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        if (!mbar_wait(bar_tempty(ab), aph ^ 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem_base + ab * ACC_STRIDE;
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait(bar_full1(s1), ph1) || !mbar_wait(bar_full2(s2), ph2)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = sbase + QP::OFF_R1 + s1 * QP::S1_BYTES;
          const uint32_t b_addr = sbase + QP::OFF_R2 + s2 * QP::B_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t adesc = smem_desc(a_addr + kk * 32, 16, 1024, 2);
            const uint64_t bdesc =
                B_MN ? smem_desc(b_addr + kk * 2048, 8192, 1024, 2) : smem_desc(b_addr + kk * 32, 16, 1024, 2);
            mma_bf16(d, adesc, bdesc, IDESC_MAIN, (kb | kk) != 0);
          }
          mma_commit(bar_empty1(s1));
          mma_commit(bar_empty2(s2));
          if (++s1 == S1) {
            s1 = 0;
            ph1 ^= 1;
          }
          if (++s2 == S2) {
            s2 = 0;
            ph2 ^= 1;
          }
          if (LORA && pend >= 0 && !issue_up(false)) { ok = false; break; }
        }
        if (!ok) break;
        if (LORA) {
          if (pend >= 0 && !issue_up(true)) { ok = false; break; }
          mma_commit(bar_lowfull(ab));
          pend = it;
        } else {
          mma_commit(bar_tfull(ab));
        }
      }
      if (ok && LORA && pend >= 0) ok = issue_up(true);
      if (!ok) {
        mma_commit(bar_drain);
        mbar_wait_drain(bar_drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------------------------------------ converters
    const int ct = threadIdx.x - Q_CONV_WARP0 * 32;
    int s1 = 0, s2 = 0;
    uint32_t ph1 = 0, ph2 = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
      const int nb = u % p.nblocks;
      for (int kb = 0; kb < p.kblocks; ++kb) {
        if (!mbar_wait(bar_full1(s1), ph1) || !mbar_wait(bar_empty2(s2), ph2 ^ 1)) { ok = false; break; }
        const uint8_t* st1 = smem + QP::OFF_R1 + s1 * QP::S1_BYTES;
        uint8_t* bdst = smem + QP::OFF_R2 + s2 * QP::B_BYTES;
        auto valid = [&](int r) {
          if (B_MN) return nb * BN + 64 * (r >> 6) < p.N;
          if (SWIGLU) return (r < 96 ? nb * 96 + r : nb * 96 + r - 96) < p.inter;
          return nb * BN + r < p.N;
        };
        convert_tasks<QF, BN, QRoles<EPI, QF>::CONV_THREADS>(ct, BN, st1 + QP::OFF_RAW, reinterpret_cast<const float*>(st1 + QP::OFF_MULT), bdst, lv,
                              valid);
        if (LORA) {  // the panel rows (K-major: B rows 192..207; MN-major: the fourth 64-column chunk), verbatim
          const uint4* ps = reinterpret_cast<const uint4*>(st1 + A_BYTES);
          uint4* pd = reinterpret_cast<uint4*>(bdst + (B_MN ? 3 * 64 * BK * 2 : BN * BK * 2));
          for (int i = ct; i < QP::PANEL_BYTES / 16; i += QRoles<EPI, QF>::CONV_THREADS) pd[i] = ps[i];
        }
        fence_proxy_async_smem();  // the bf16 tile, written by these threads, is read by the tensor cores
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(bar_full2(s2));
          mbar_arrive(bar_empty1(s1));
        }
        if (++s1 == S1) {
          s1 = 0;
          ph1 ^= 1;
        }
        if (++s2 == S2) {
          s2 = 0;
          ph2 ^= 1;
        }
      }
    }
  }
}

template <bool B_MN, bool LORA, int EPI, int QF>
__global__ void __launch_bounds__(Q_THREADS, 1)
    grouped_gemm_q_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_raw,
                          const __grid_constant__ CUtensorMap tm_mult, const __grid_constant__ CUtensorMap tm_p,
                          const __grid_constant__ CUtensorMap tm_u, const Params p) {
  using QP = QPlan<B_MN, QF>;
  using R = QRoles<EPI, QF>;
  constexpr int S1 = QP::S1, S2 = QP::S2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const uint32_t bar0 = sbase + QP::OFF_BAR;
  auto bar_full1 = [&](int s) { return bar0 + 8u * s; };
  auto bar_empty1 = [&](int s) { return bar0 + 8u * (S1 + s); };
  auto bar_full2 = [&](int s) { return bar0 + 8u * (2 * S1 + s); };
  auto bar_empty2 = [&](int s) { return bar0 + 8u * (2 * S1 + S2 + s); };
  const uint32_t bar1 = bar0 + 8u * (2 * S1 + 2 * S2);
  auto bar_tfull = [&](int b) { return bar1 + 8u * b; };
  auto bar_tempty = [&](int b) { return bar1 + 8u * (2 + b); };
  auto bar_lowfull = [&](int b) { return bar1 + 8u * (4 + b); };
  const uint32_t bar_lowready = bar1 + 8u * 6;
  const uint32_t bar_ufull = bar1 + 8u * 7;
  const uint32_t bar_uempty = bar1 + 8u * 8;
  const uint32_t bar_drain = bar1 + 8u * 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + QP::OFF_TMEM);
  float* lv = reinterpret_cast<float*>(smem + QP::OFF_LUT);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S1; ++s) {
      mbar_init(bar_full1(s), 1);
      mbar_init(bar_empty1(s), R::CONV_WARPS + 1);  // each converter warp has read the codes; the MMAs the x tile
    }
    for (int s = 0; s < S2; ++s) {
      mbar_init(bar_full2(s), R::CONV_WARPS);
      mbar_init(bar_empty2(s), 1);
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
    fence_barrier_init();
  }
  if (QF == QF_NF4 && threadIdx.x < 16) lv[threadIdx.x] = kNF4Levels[threadIdx.x];
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total = (*p.tiles) * p.nblocks;

  if (warp < R::EPI_WARP0) {
    if (R::CONV_WARPS == 10) {
      asm volatile("setmaxnreg.dec.sync.aligned.u32 112;");
    } else {
      asm volatile("setmaxnreg.dec.sync.aligned.u32 80;");
    }
    q_mainloop_roles<B_MN, LORA, EPI, QF>(tm_x, tm_raw, tm_mult, tm_p, tm_u, p, smem, sbase, tmem_base, total, warp,
                                          lane);
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 176;");
    // ------------------------------------------------------------------------------------------ epilogue
    const uint32_t bar1 = sbase + QP::OFF_BAR + 8u * (2 * S1 + 2 * S2);
    const int qd = warp & 3;
    const int half0 = R::EPI_HALVES == 1 ? (warp - R::EPI_WARP0) >> 2 : 0;
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ++it) {
      const int ab = it & 1;
      for (int h = 0; h < R::EPI_HALVES && ok; ++h)
        ok = epilogue_unit<EPI, LORA, false>(p, u, it, 0, smem + QP::OFF_LOW, tmem_base, qd, half0 + h, lane,
                                             bar1 + 8u * (4 + ab), bar1 + 8u * 6, bar1 + 8u * ab,
                                             bar1 + 8u * (2 + ab));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <bool B_MN, bool LORA, int EPI, int QF>
static int launch_q(const CUtensorMap& tx, const CUtensorMap& traw, const CUtensorMap& tmult, const CUtensorMap& tp,
                    const CUtensorMap& tu, const Params& prm, int grid, cudaStream_t s) {
  auto kern = grouped_gemm_q_kernel<B_MN, LORA, EPI, QF>;
  static bool configured = false;
  if (!configured) {
    // setmaxnreg.inc draws on the registers the block was launched with: the splits of QRoles need exactly 128
    // per thread at launch, else the epilogue's increase could never be granted
    cudaFuncAttributes attr;
    if (cudaFuncGetAttributes(&attr, kern) != cudaSuccess || attr.numRegs != 128 ||
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, QPlan<B_MN, QF>::SMEM_BYTES) !=
            cudaSuccess) {
      cudaGetLastError();
      return MEEP2B_ERR_LAUNCH;
    }
    configured = true;
  }
  kern<<<grid, Q_THREADS, QPlan<B_MN, QF>::SMEM_BYTES, s>>>(tx, traw, tmult, tp, tu, prm);
  return launch_status();
}

template <int QF>
static int dispatch_q(bool mn, bool lora, int epi, const CUtensorMap& tx, const CUtensorMap& traw,
                      const CUtensorMap& tmult, const CUtensorMap& tp, const CUtensorMap& tu, const Params& prm,
                      int grid, cudaStream_t s) {
#define MEEP2B_Q(MN, L, EP) launch_q<MN, L, EP, QF>(tx, traw, tmult, tp, tu, prm, grid, s)
  switch (epi) {
    case MEEP2B_EPI_PLAIN:
      if (mn) return lora ? MEEP2B_Q(true, true, 0) : MEEP2B_Q(true, false, 0);
      return lora ? MEEP2B_Q(false, true, 0) : MEEP2B_Q(false, false, 0);
    case MEEP2B_EPI_SWIGLU:
      return lora ? MEEP2B_Q(false, true, 1) : MEEP2B_Q(false, false, 1);
    default:
      if (mn) return lora ? MEEP2B_Q(true, true, 2) : MEEP2B_Q(true, false, 2);
      return lora ? MEEP2B_Q(false, true, 2) : MEEP2B_Q(false, false, 2);
  }
#undef MEEP2B_Q
}

// The raw-code tensor map and the launch of a quantised product; the x, panel and up maps and Params come from
// the bf16 path's set-up. Requires k and n multiples of 64 (whole NF4 blocks and 64-column groups).
static int launch_quantized(const meep2b_product* a, const CUtensorMap& tx, const CUtensorMap& tp,
                            const CUtensorMap& tu, const Params& prm, int grid, cudaStream_t s) {
  const uint64_t K = a->k, N = a->n, E = a->experts;
  const int dt = a->weight_dtype;
  const int qf = dt == MEEP2B_NF4 ? QF_NF4 : dt == MEEP2B_E4M3 ? QF_E4M3 : QF_E4M3_BLOCKS;
  if (K % 64 || N % 64) return MEEP2B_ERR_UNSUPPORTED;
  if (qf != QF_E4M3 && a->wscale == nullptr) return MEEP2B_ERR_SHAPE;
  if (qf != QF_E4M3 && a->scale != nullptr) return MEEP2B_ERR_UNSUPPORTED;  // the scale lives in the blocks
  const bool swiglu = a->epilogue == MEEP2B_EPI_SWIGLU;
  const uint64_t bpe2 = qf == QF_NF4 ? 1 : 2;  // code bytes per two weights
  // the stored matrix of each expert: rows x cols, cols contiguous
  const uint64_t srows = a->b_mn ? K : N, scols = a->b_mn ? N : K;
  CUtensorMap traw;
  {
    const uint64_t dims[3] = {scols * bpe2 / 2, srows, E};
    const uint64_t strides[2] = {scols * bpe2 / 2, srows * scols * bpe2 / 2};
    uint32_t box[3];
    box[0] = static_cast<uint32_t>(64 * bpe2 / 2);  // one 64-weight group of a row
    box[1] = a->b_mn ? static_cast<uint32_t>(BK) : (swiglu ? 96u : static_cast<uint32_t>(BN));
    box[2] = 1;
    MEEP2B_TRY(encode_tiled(&traw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, a->weight, dims, strides, box,
                            qf == QF_NF4 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B));
  }
  CUtensorMap tmult = traw;
  if (qf != QF_E4M3) {  // the multipliers, (experts, cols/64, rows) float32
    const uint64_t dims[3] = {srows, scols / 64, E};
    const uint64_t strides[2] = {srows * 4, (scols / 64) * srows * 4};
    const uint32_t box[3] = {a->b_mn ? 64u : (swiglu ? 96u : static_cast<uint32_t>(BN)), a->b_mn ? 3u : 1u, 1u};
    MEEP2B_TRY(encode_tiled(&tmult, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, a->wscale, dims, strides, box,
                            CU_TENSOR_MAP_SWIZZLE_NONE));
  }
  const bool mn = a->b_mn != 0, lora = a->panel != nullptr;
  const int epi = a->epilogue;
  if (qf == QF_NF4) return dispatch_q<QF_NF4>(mn, lora, epi, tx, traw, tmult, tp, tu, prm, grid, s);
  if (qf == QF_E4M3) return dispatch_q<QF_E4M3>(mn, lora, epi, tx, traw, tmult, tp, tu, prm, grid, s);
  return dispatch_q<QF_E4M3_BLOCKS>(mn, lora, epi, tx, traw, tmult, tp, tu, prm, grid, s);
}

// The quantised product on CTA pairs (tcgen05 cta_group::2), for stacks read K-major (the forward products).
//
// Included by grouped_gemm.cu after grouped_gemm_q.cuh (namespace meep2b::gemm). A work unit is 256 rows of one
// expert by 192 columns, as in the bf16 pair kernel: CTA r holds rows 128 r .. 128 r + 127 of the x tile and its
// half of the 208-row B tile (the second CTA's last 16 rows are the rank panel). Each CTA's converters dequantise
// only its own half of B, so an SM converts and stages ~104 rows per k-step instead of 192: the shared-memory
// traffic that bounds the one-CTA fused product (~114 KB per k-step) drops to ~71 KB.
//
// Per CTA, 16 warps: warp 0 the TMA producer (the x tile by a pair load completing on the leader's barrier; the raw
// codes, multipliers and panel of this CTA's rows by local loads on a local barrier), warp 1 the leader's MMA issuer,
// warps 2-11 converters (this CTA's B rows -> bf16, 128-byte swizzle; arrivals on the leader's barrier), warps 12-15
// the epilogue of this CTA's 128 rows. Registers as in the one-CTA quantised kernel (setmaxnreg 112 / 176).

template <bool LORA, int QF>
struct QPairPlan {
  static constexpr int RAW_ROW = QF == QF_NF4 ? 32 : 64;
  static constexpr int B_ROWS = LORA ? PAIR_B_ROWS : BN / 2;     // 104 or 96 rows of B per CTA
  static constexpr int RAW_BYTES = ((B_ROWS * RAW_ROW + 1023) / 1024) * 1024;
  static constexpr int MULT_BYTES = QF == QF_E4M3 ? 0 : 512;      // B_ROWS floats
  static constexpr int PANEL_BYTES = RP * BK * 2;                  // the second CTA's 16 panel rows
  static constexpr int OFF_PANEL = A_BYTES;
  static constexpr int OFF_RAW = A_BYTES + PANEL_BYTES;
  static constexpr int OFF_MULT = OFF_RAW + RAW_BYTES;
  static constexpr int S1_BYTES = ((OFF_MULT + MULT_BYTES + 1023) / 1024) * 1024;
  static constexpr int B_BYTES = PAIR_B_ROWS * BK * 2;             // 104 rows of 128 bytes (13 KB)
  static constexpr int U_BYTES_P = 4096;
  static constexpr int S2 = 6;
  static constexpr int FWD_BATCH = 1;  // converted stages the forwarder waits for before passing them on (measured best)
  static constexpr int BUDGET = 232448 - 1024 - 1024 - 1024;
  static constexpr int S1_FIT = (BUDGET - S2 * B_BYTES - U_BYTES_P - LOW_BYTES) / S1_BYTES;
  static constexpr int S1 = S1_FIT > 6 ? 6 : S1_FIT;
  static constexpr int OFF_R1 = 0;
  static constexpr int OFF_R2 = OFF_R1 + S1 * S1_BYTES;
  static constexpr int OFF_U = OFF_R2 + S2 * B_BYTES;
  static constexpr int OFF_LOW = OFF_U + U_BYTES_P;
  static constexpr int OFF_LUT = OFF_LOW + LOW_BYTES;
  static constexpr int OFF_BAR = OFF_LUT + 1024;
  static constexpr int NUM_BARS = 3 * S1 + 3 * S2 + 10;
  static constexpr int OFF_TMEM = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_TMEM + 16 + 1024;
  static_assert(S1 >= 3, "the quantised pair ring needs three stages");
  static_assert(SMEM_BYTES <= 232448, "quantised pair plan exceeds 227 KB");
  static_assert(S1_BYTES % 1024 == 0 && B_BYTES % 1024 == 0 && OFF_R2 % 1024 == 0 && OFF_U % 1024 == 0 &&
                    OFF_LOW % 1024 == 0, "swizzled tiles need 1 KB alignment");
};

struct QPairMaps {
  CUtensorMap x;     // (k, rows) box 64 x 128, 128-byte swizzle
  CUtensorMap r104;  // raw codes (k bytes, n, E), box (64-weight group) x 104 / 96 / 88 / 8 rows
  CUtensorMap r96;
  CUtensorMap r88;
  CUtensorMap r8;
  CUtensorMap m104;  // multipliers (n, k/64, E) float32, box 104 / 96 / 88 / 8 x 1
  CUtensorMap m96;
  CUtensorMap m88;
  CUtensorMap m8;
  CUtensorMap p16;   // panel (k, 16, E) box 64 x 16
  CUtensorMap u96;   // up (16, n, E) box 16 x 96, 32-byte swizzle
};

// The B rows of this CTA for a unit: up to two runs of stored rows (first run: `n1` rows from stored row `s1`,
// second: `n2` rows from `s2`), valid below `lim1` / `lim2` (run-relative indices of rows past the stack's end are
// zero-filled); with the adapters the second CTA's last 16 rows are the panel.
struct QPairRows {
  int s1, n1, lim1, s2, n2, lim2;
};

template <bool LORA, int EPI>
__device__ __forceinline__ QPairRows qpair_rows(const Params& p, int nb, uint32_t rank) {
  QPairRows r{};
  if (EPI == MEEP2B_EPI_SWIGLU) {
    const int g0 = nb * 96, glim = p.inter - g0;  // gate / up rows j of this block valid while j < glim
    if (!LORA) {
      r.s1 = rank == 0 ? g0 : p.inter + g0, r.n1 = 96, r.lim1 = glim;
      r.n2 = 0;
    } else if (rank == 0) {
      r.s1 = g0, r.n1 = 96, r.lim1 = glim;                   // gate 0..95
      r.s2 = p.inter + g0, r.n2 = 8, r.lim2 = glim;          // up 0..7
    } else {
      r.s1 = p.inter + g0 + 8, r.n1 = 88, r.lim1 = glim - 8;  // up 8..95
      r.n2 = 0;
    }
  } else {
    const int n0 = nb * BN;
    if (!LORA) {
      r.s1 = n0 + 96 * static_cast<int>(rank), r.n1 = 96;
    } else {
      r.s1 = rank == 0 ? n0 : n0 + 104, r.n1 = rank == 0 ? 104 : 88;
    }
    r.lim1 = p.N - r.s1;
    r.n2 = 0;
  }
  return r;
}

template <bool LORA, int EPI, int QF>
__device__ __forceinline__ void qpair_mainloop_roles(const QPairMaps& m, const Params& p, uint8_t* smem,
                                                     uint32_t sbase, uint32_t tmem_base, int total, int warp,
                                                     int lane, uint32_t rank, int pair_id, int pairs) {
  using QP = QPairPlan<LORA, QF>;
  constexpr int S1 = QP::S1, S2 = QP::S2;
  const uint32_t bar0 = sbase + QP::OFF_BAR;
  auto bar_fulla = [&](int s) { return bar0 + 8u * s; };             // leader's: x tiles of both CTAs
  auto bar_fullr = [&](int s) { return bar0 + 8u * (S1 + s); };      // local: codes, multipliers, panel
  auto bar_empty1 = [&](int s) { return bar0 + 8u * (2 * S1 + s); }; // local
  auto bar_full2 = [&](int s) { return bar0 + 8u * (3 * S1 + s); };  // leader's: both halves converted
  auto bar_empty2 = [&](int s) { return bar0 + 8u * (3 * S1 + S2 + s); };
  const uint32_t bar1 = bar0 + 8u * (3 * S1 + 2 * S2);
  auto bar_conv = [&](int s) { return bar1 + 8u * (10 + s); };  // second CTA: its own converters done (local)
  auto bar_tfull = [&](int b) { return bar1 + 8u * b; };
  auto bar_tempty = [&](int b) { return bar1 + 8u * (2 + b); };
  auto bar_lowfull = [&](int b) { return bar1 + 8u * (4 + b); };
  const uint32_t bar_lowready = bar1 + 8u * 6;
  const uint32_t bar_ufull = bar1 + 8u * 7;
  const uint32_t bar_uempty = bar1 + 8u * 8;
  const uint32_t bar_drain = bar1 + 8u * 9;
  const float* lv = reinterpret_cast<const float*>(smem + QP::OFF_LUT);
  constexpr int BPE = QF == QF_NF4 ? 1 : 2;  // code bytes are (weights * BPE) / 2

  if (warp == 0) {
    // ------------------------------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint32_t raw_tx =
          static_cast<uint32_t>(QP::RAW_ROW * (LORA && rank == 1 ? 88 : QP::B_ROWS)) +
          (QF == QF_E4M3 ? 0u : static_cast<uint32_t>(4 * (LORA && rank == 1 ? 88 : QP::B_ROWS))) +
          (LORA && rank == 1 ? static_cast<uint32_t>(QP::PANEL_BYTES) : 0u);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t last_parity[S1];
      bool issued[S1];
      for (int s = 0; s < S1; ++s) issued[s] = false, last_parity[s] = 0;
      bool ok = true;
      int it = 0;
      int pu = -1, pu_nb = 0, pu_e = 0;
      auto load_u = [&]() -> bool {
        if (!mbar_wait(bar_uempty, (pu & 1) ^ 1)) return false;
        if (rank == 0) mbar_arrive_expect_tx(bar_ufull, 2 * (BN / 2) * RP * 2);
        const int urow = EPI == MEEP2B_EPI_SWIGLU ? (rank == 0 ? pu_nb * 96 : p.inter + pu_nb * 96)
                                                  : pu_nb * BN + 96 * static_cast<int>(rank);
        tma_load_3d_pair(sbase + QP::OFF_U, &m.u96, map_to_rank(bar_ufull, 0), 0, urow, pu_e);
        pu = -1;
        return true;
      };
      auto box = [&](int n, bool raw) -> const CUtensorMap* {
        if (raw) return n == 104 ? &m.r104 : n == 96 ? &m.r96 : n == 88 ? &m.r88 : &m.r8;
        return n == 104 ? &m.m104 : n == 96 ? &m.m96 : n == 88 ? &m.m88 : &m.m8;
      };
      for (int u = pair_id; u < total && ok; u += pairs, ++it) {
        const int t = u / p.nblocks, nb = u - t * p.nblocks;
        const int e = p.tile_expert[t], row0 = p.tile_row[t] + 128 * static_cast<int>(rank);
        const QPairRows rows = qpair_rows<LORA, EPI>(p, nb, rank);
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait(bar_empty1(stage), phase ^ 1)) { ok = false; break; }
          const uint32_t s_dst = sbase + QP::OFF_R1 + stage * QP::S1_BYTES;
          if (rank == 0) mbar_arrive_expect_tx(bar_fulla(stage), 2 * A_BYTES);
          tma_load_2d_pair(s_dst, &m.x, map_to_rank(bar_fulla(stage), 0), kb * BK, row0);
          const uint32_t fr = bar_fullr(stage);
          mbar_arrive_expect_tx(fr, raw_tx);
          const int x0 = kb * BK * BPE / 2;
          tma_load_3d(s_dst + QP::OFF_RAW, box(rows.n1, true), fr, x0, rows.s1, e);
          if (QF != QF_E4M3) tma_load_3d(s_dst + QP::OFF_MULT, box(rows.n1, false), fr, rows.s1, kb, e);
          if (rows.n2 > 0) {
            tma_load_3d(s_dst + QP::OFF_RAW + rows.n1 * QP::RAW_ROW, box(rows.n2, true), fr, x0, rows.s2, e);
            if (QF != QF_E4M3) tma_load_3d(s_dst + QP::OFF_MULT + 4 * rows.n1, box(rows.n2, false), fr, rows.s2, kb, e);
          }
          if (LORA && rank == 1) tma_load_3d(s_dst + QP::OFF_PANEL, &m.p16, fr, kb * BK, 0, e);
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
        for (int s = 0; s < S1; ++s) {
          if (!issued[s]) continue;
          mbar_wait_drain(bar_fullr(s), last_parity[s]);
          if (rank == 0) mbar_wait_drain(bar_fulla(s), last_parity[s]);
        }
      }
    }
  } else if (warp == 1 && rank == 1) {
    // ------------------------------------------------------------------------------------------ forwarder
    // The second CTA's converter warps arrive on a local barrier (a release at CTA scope); this thread passes the
    // completed stages on to the leader's barriers in batches, under one cluster-scope fence followed by relaxed
    // arrives (a release pattern per arrive). A cluster-scope release from every converter warp, or one per stage,
    // stalls on the memory barrier it implies (measured: the pair's rate rose from 390 to ~600 TFLOP/s with e4m3
    // codes as the per-warp releases became batched ones).
    if (lane == 0) {
      const int units = pair_id < total ? (total - 1 - pair_id) / pairs + 1 : 0;
      const int64_t stages = static_cast<int64_t>(units) * p.kblocks;
      int s2 = 0;
      uint32_t ph2 = 0;
      bool ok = true;
      for (int64_t done = 0; done < stages && ok;) {
        // wait for a batch of stages (fewer at the end), then take any further ones already converted; each is
        // observed before the arrives below
        const int batch = static_cast<int>(stages - done < QP::FWD_BATCH ? stages - done : QP::FWD_BATCH);
        int n = 0;
        int t = s2;
        uint32_t pt = ph2;
        while (n < S2 && done + n < stages) {
          if (n < batch) {
            if (!mbar_wait(bar_conv(t), pt)) {
              ok = false;
              break;
            }
          } else if (!mbar_test(bar_conv(t), pt)) {
            break;
          }
          ++n;
          if (++t == S2) {
            t = 0;
            pt ^= 1;
          }
        }
        if (!ok) break;
        fence_cluster();
        for (int i = 0; i < n; ++i) {
          mbar_arrive_remote_relaxed(bar_full2(s2), 0);
          if (++s2 == S2) {
            s2 = 0;
            ph2 ^= 1;
          }
        }
        done += n;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------------------ MMA issuer (leader)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t IDESC_MAIN = idesc_bf16(256, LORA ? BN + RP : BN, false, false);
      constexpr uint32_t IDESC_UP = idesc_bf16(256, BN, false, false);
      int s1 = 0, s2 = 0;
      uint32_t ph1 = 0, ph2 = 0;
      bool ok = true;
      int it = 0;
      int pend = -1;
      auto issue_up = [&](bool block) -> bool {
        const uint32_t par = static_cast<uint32_t>(pend) & 1;
        if (block) {
          if (!mbar_wait_cluster(bar_lowready, par) || !mbar_wait(bar_ufull, par)) return false;
        } else if (!mbar_test_cluster(bar_lowready, par) || !mbar_test(bar_ufull, par)) {
          return true;
        }
        tc_fence_after();
        const uint32_t dp = tmem_base + (pend & 1) * ACC_STRIDE;
        const uint32_t low_addr = sbase + QP::OFF_LOW;
        const uint64_t bdesc = smem_desc(sbase + QP::OFF_U, 16, 256, 6);
        mma_bf16_pair(dp, smem_desc(low_addr, 16, 256, 6), bdesc, IDESC_UP, 1);
        mma_bf16_pair(dp, smem_desc(low_addr + BM * RP * 2, 16, 256, 6), bdesc, IDESC_UP, 1);
        mma_commit_pair(bar_uempty);
        mma_commit_pair(bar_tfull(pend & 1));
        pend = -1;
        return true;
      };
      for (int u = pair_id; u < total && ok; u += pairs, ++it) {
        const int ab = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        if (!mbar_wait_cluster(bar_tempty(ab), aph ^ 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem_base + ab * ACC_STRIDE;
        for (int kb = 0; kb < p.kblocks; ++kb) {
          // the x tiles (TMA) and both CTAs' converted halves (generic writes released at cluster scope)
          if (!mbar_wait(bar_fulla(s1), ph1) || !mbar_wait_cluster(bar_full2(s2), ph2)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = sbase + QP::OFF_R1 + s1 * QP::S1_BYTES;
          const uint32_t b_addr = sbase + QP::OFF_R2 + s2 * QP::B_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_bf16_pair(d, smem_desc(a_addr + kk * 32, 16, 1024, 2), smem_desc(b_addr + kk * 32, 16, 1024, 2),
                          IDESC_MAIN, (kb | kk) != 0);
          mma_commit_pair(bar_empty1(s1));
          mma_commit_pair(bar_empty2(s2));
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
  } else {
    // ------------------------------------------------------------------------------------------ converters
    const int ct = threadIdx.x - Q_CONV_WARP0 * 32;
    int s1 = 0, s2 = 0;
    uint32_t ph1 = 0, ph2 = 0;
    bool ok = true;
    for (int u = pair_id; u < total && ok; u += pairs) {
      const int nb = u % p.nblocks;
      const QPairRows rows = qpair_rows<LORA, EPI>(p, nb, rank);
      const int conv_rows = rows.n1 + rows.n2;
      // the validity of B row r (rows past the stack's end are zero-filled)
      auto valid = [&](int r) { return r < rows.n1 ? r < rows.lim1 : r - rows.n1 < rows.lim2; };
      for (int kb = 0; kb < p.kblocks; ++kb) {
        if (!mbar_wait(bar_fullr(s1), ph1) || !mbar_wait(bar_empty2(s2), ph2 ^ 1)) { ok = false; break; }
        const uint8_t* st1 = smem + QP::OFF_R1 + s1 * QP::S1_BYTES;
        uint8_t* bdst = smem + QP::OFF_R2 + s2 * QP::B_BYTES;
        convert_tasks<QF, QP::B_ROWS, QRoles<EPI, QF>::CONV_THREADS>(ct, conv_rows, st1 + QP::OFF_RAW,
                                      reinterpret_cast<const float*>(st1 + QP::OFF_MULT), bdst, lv, valid);
        if (LORA && rank == 1) {  // the panel: B rows 88..103 of the second CTA, verbatim (same swizzle phase)
          const uint4* ps = reinterpret_cast<const uint4*>(st1 + QP::OFF_PANEL);
          uint4* pd = reinterpret_cast<uint4*>(bdst + 88 * 128);
          for (int i = ct; i < QP::PANEL_BYTES / 16; i += QRoles<EPI, QF>::CONV_THREADS) pd[i] = ps[i];
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(rank == 0 ? bar_full2(s2) : bar_conv(s2));
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

template <bool LORA, int EPI, int QF>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Q_THREADS, 1)
    grouped_gemm_qpair_kernel(const __grid_constant__ QPairMaps m, const Params p) {
  using QP = QPairPlan<LORA, QF>;
  constexpr int S1 = QP::S1, S2 = QP::S2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair_id = static_cast<int>(cluster_id_x()), pairs = static_cast<int>(num_clusters_x());
  const uint32_t bar0 = sbase + QP::OFF_BAR;
  const uint32_t bar1 = bar0 + 8u * (3 * S1 + 2 * S2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + QP::OFF_TMEM);
  float* lv = reinterpret_cast<float*>(smem + QP::OFF_LUT);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S1; ++s) {
      mbar_init(bar0 + 8u * s, 1);                      // x tiles (leader's)
      mbar_init(bar0 + 8u * (S1 + s), 1);               // codes, multipliers, panel (local)
      mbar_init(bar0 + 8u * (2 * S1 + s), QRoles<EPI, QF>::CONV_WARPS + 1);  // the converters and the pair's MMAs
    }
    for (int s = 0; s < S2; ++s) {
      // the leader's converter warps and the second CTA's forwarder (leader's barrier)
      mbar_init(bar0 + 8u * (3 * S1 + s), QRoles<EPI, QF>::CONV_WARPS + 1);
      mbar_init(bar0 + 8u * (3 * S1 + S2 + s), 1);
      mbar_init(bar1 + 8u * (10 + s), QRoles<EPI, QF>::CONV_WARPS);  // the second CTA's converter warps (local)
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar1 + 8u * b, 1);
      mbar_init(bar1 + 8u * (2 + b), 512);
      mbar_init(bar1 + 8u * (4 + b), 1);
    }
    mbar_init(bar1 + 8u * 6, 256);
    mbar_init(bar1 + 8u * 7, 1);
    mbar_init(bar1 + 8u * 8, 1);
    mbar_init(bar1 + 8u * 9, 1);
    fence_barrier_init();
  }
  if (QF == QF_NF4 && threadIdx.x < 16) lv[threadIdx.x] = kNF4Levels[threadIdx.x];
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total = (*p.tiles) * p.nblocks;

  static_assert(QRoles<EPI, QF>::CONV_WARPS == 10, "the pair kernel runs the forward products' roles");
  if (warp < QRoles<EPI, QF>::EPI_WARP0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 112;");
    qpair_mainloop_roles<LORA, EPI, QF>(m, p, smem, sbase, tmem_base, total, warp, lane, rank, pair_id, pairs);
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 176;");
    const int qd = warp & 3;
    int it = 0;
    bool ok = true;
    for (int u = pair_id; u < total && ok; u += pairs, ++it) {
      const int ab = it & 1;
      for (int half = 0; half < 2 && ok; ++half)
        ok = epilogue_unit<EPI, LORA, true>(p, u, it, 128 * static_cast<int>(rank), smem + QP::OFF_LOW, tmem_base,
                                            qd, half, lane, bar1 + 8u * (4 + ab), bar1 + 8u * 6, bar1 + 8u * ab,
                                            bar1 + 8u * (2 + ab));
    }
  }

  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

template <bool LORA, int EPI, int QF>
static int launch_qpair(const QPairMaps& maps, const Params& prm, int grid, cudaStream_t s) {
  auto kern = grouped_gemm_qpair_kernel<LORA, EPI, QF>;
  static bool configured = false;
  if (!configured) {
    cudaFuncAttributes attr;  // the setmaxnreg split needs exactly 128 registers per thread at launch
    if (cudaFuncGetAttributes(&attr, kern) != cudaSuccess || attr.numRegs != 128 ||
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, QPairPlan<LORA, QF>::SMEM_BYTES) !=
            cudaSuccess) {
      cudaGetLastError();
      return MEEP2B_ERR_LAUNCH;
    }
    configured = true;
  }
  kern<<<grid, Q_THREADS, QPairPlan<LORA, QF>::SMEM_BYTES, s>>>(maps, prm);
  return launch_status();
}

template <int QF>
static int dispatch_qpair(bool lora, int epi, const QPairMaps& maps, const Params& prm, int grid, cudaStream_t s) {
  if (epi == MEEP2B_EPI_SWIGLU)
    return lora ? launch_qpair<true, 1, QF>(maps, prm, grid, s) : launch_qpair<false, 1, QF>(maps, prm, grid, s);
  if (epi == MEEP2B_EPI_PLAIN)
    return lora ? launch_qpair<true, 0, QF>(maps, prm, grid, s) : launch_qpair<false, 0, QF>(maps, prm, grid, s);
  return MEEP2B_ERR_UNSUPPORTED;
}

// A quantised K-major product on CTA pairs (block_m 256): the tensor maps and the launch.
static int launch_quantized_pair(const meep2b_product* a, const CUtensorMap& tx, const Params& prm, int sms,
                                 cudaStream_t s) {
  const uint64_t K = a->k, N = a->n, E = a->experts;
  const int dt = a->weight_dtype;
  const int qf = dt == MEEP2B_NF4 ? QF_NF4 : dt == MEEP2B_E4M3 ? QF_E4M3 : QF_E4M3_BLOCKS;
  if (a->b_mn || K % 64 || N % 64) return MEEP2B_ERR_UNSUPPORTED;
  if (a->epilogue != MEEP2B_EPI_SWIGLU && a->epilogue != MEEP2B_EPI_PLAIN) return MEEP2B_ERR_UNSUPPORTED;
  if (qf != QF_E4M3 && a->wscale == nullptr) return MEEP2B_ERR_SHAPE;
  if (qf != QF_E4M3 && a->scale != nullptr) return MEEP2B_ERR_UNSUPPORTED;
  const bool lora = a->panel != nullptr;
  const uint64_t bpe2 = qf == QF_NF4 ? 1 : 2;
  QPairMaps maps;
  maps.x = tx;
  const uint32_t heights[4] = {104, 96, 88, 8};
  CUtensorMap* raws[4] = {&maps.r104, &maps.r96, &maps.r88, &maps.r8};
  CUtensorMap* mults[4] = {&maps.m104, &maps.m96, &maps.m88, &maps.m8};
  for (int i = 0; i < 4; ++i) {
    const uint64_t dims[3] = {K * bpe2 / 2, N, E};
    const uint64_t strides[2] = {K * bpe2 / 2, N * K * bpe2 / 2};
    const uint32_t box[3] = {static_cast<uint32_t>(64 * bpe2 / 2), heights[i], 1};
    MEEP2B_TRY(encode_tiled(raws[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, a->weight, dims, strides, box,
                            qf == QF_NF4 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B));
    if (qf != QF_E4M3) {
      const uint64_t md[3] = {N, K / 64, E};
      const uint64_t ms[2] = {N * 4, (K / 64) * N * 4};
      const uint32_t mb[3] = {heights[i], 1, 1};
      MEEP2B_TRY(encode_tiled(mults[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, a->wscale, md, ms, mb,
                              CU_TENSOR_MAP_SWIZZLE_NONE));
    } else {
      *mults[i] = *raws[i];
    }
  }
  maps.p16 = maps.u96 = tx;
  if (lora) {
    const uint64_t pd[3] = {K, RP, E};
    const uint64_t ps[2] = {K * 2, RP * K * 2};
    const uint32_t pb[3] = {64, RP, 1};
    MEEP2B_TRY(encode_tiled(&maps.p16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a->panel, pd, ps, pb,
                            CU_TENSOR_MAP_SWIZZLE_128B));
    const uint64_t ud[3] = {RP, N, E};
    const uint64_t us[2] = {RP * 2, N * RP * 2};
    const uint32_t ubx[3] = {RP, 96, 1};
    MEEP2B_TRY(encode_tiled(&maps.u96, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a->up, ud, us, ubx,
                            CU_TENSOR_MAP_SWIZZLE_32B));
  }
  const int64_t units = a->max_tiles * prm.nblocks;
  const int pairs_max = sms / 2;
  const int64_t pairs = units < pairs_max ? (units > 0 ? units : 1) : pairs_max;
  const int grid = static_cast<int>(2 * pairs);
  if (qf == QF_NF4) return dispatch_qpair<QF_NF4>(lora, a->epilogue, maps, prm, grid, s);
  if (qf == QF_E4M3) return dispatch_qpair<QF_E4M3>(lora, a->epilogue, maps, prm, grid, s);
  return dispatch_qpair<QF_E4M3_BLOCKS>(lora, a->epilogue, maps, prm, grid, s);
}

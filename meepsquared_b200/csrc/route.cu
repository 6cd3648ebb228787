// Routing kernels of the expert layer: the stable counting sort of the expert ids (histogram, offset table,
// scatter), the gather of hidden rows into expert order, the weighted un-permute and its backward, and the tile
// map of the grouped product. All HBM- or latency-bound integer and byte work: coalesced 16-byte accesses, no
// tensor cores.
//
// Replaces _moe._routed_forward's sort / histc / cumsum / gather / weighted sum (meepsquared/_moe.py:75-87,
// 123-126) and _grouped.tile_map (meepsquared/_grouped.py:88-103).
#include <mutex>

#include "common.cuh"
#include "host.hpp"

namespace meep2b {

constexpr int kRouteChunk = 4096;   // assignments per CTA of the histogram and scatter passes
constexpr int kRouteThreads = 256;  // 8 warps: a round of the scatter places 256 assignments
constexpr int kMaxBuckets = 1025;   // experts + 1 (the sentinel bucket)

__device__ __forceinline__ int bucket_of(int64_t id, int experts) {
  return (id >= 0 && id < experts) ? static_cast<int>(id) : experts;
}

// Per-CTA bucket counts of its chunk: counts[block * buckets + b].
__global__ void __launch_bounds__(kRouteThreads) route_histogram(const int64_t* __restrict__ ids, int64_t n,
                                                                 int experts, int* __restrict__ counts) {
  extern __shared__ int hist[];
  const int buckets = experts + 1;
  for (int b = threadIdx.x; b < buckets; b += blockDim.x) hist[b] = 0;
  __syncthreads();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kRouteChunk;
  const int64_t end = min(base + kRouteChunk, n);
  for (int64_t i = base + threadIdx.x; i < end; i += blockDim.x) atomicAdd(&hist[bucket_of(ids[i], experts)], 1);
  __syncthreads();
  for (int b = threadIdx.x; b < buckets; b += blockDim.x) counts[static_cast<int64_t>(blockIdx.x) * buckets + b] = hist[b];
}

// One CTA: turns the per-CTA counts into per-CTA starting positions (bucket-major, then CTA order: this is what
// makes the sort stable) and writes the inclusive int32 offsets of the real experts.
__global__ void __launch_bounds__(1024) route_scan(int* __restrict__ counts, int blocks, int experts,
                                                   int32_t* __restrict__ offsets) {
  __shared__ int totals[kMaxBuckets];
  __shared__ int starts[kMaxBuckets];
  const int buckets = experts + 1;
  for (int b = threadIdx.x; b < buckets; b += blockDim.x) {
    int s = 0;
    for (int k = 0; k < blocks; ++k) s += counts[static_cast<int64_t>(k) * buckets + b];
    totals[b] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int b = 0; b < buckets; ++b) {
      starts[b] = run;
      run += totals[b];
    }
  }
  __syncthreads();
  for (int b = threadIdx.x; b < buckets; b += blockDim.x) {
    int run = starts[b];
    for (int k = 0; k < blocks; ++k) {
      const int64_t at = static_cast<int64_t>(k) * buckets + b;
      const int c = counts[at];
      counts[at] = run;
      run += c;
    }
    if (b < experts) offsets[b] = starts[b] + totals[b];
  }
}

// Places each assignment of the CTA's chunk at its stable position: CTA start of its bucket + the number of
// earlier assignments of the same bucket in the chunk. Rounds of 256: within a warp the rank comes from
// __match_any_sync, across the warps of a round from per-warp bucket counts.
__global__ void __launch_bounds__(kRouteThreads) route_scatter(const int64_t* __restrict__ ids, int64_t n,
                                                               int experts, const int* __restrict__ starts,
                                                               int64_t* __restrict__ perm,
                                                               int64_t* __restrict__ ids_g,
                                                               int64_t* __restrict__ inverse) {
  extern __shared__ int smem[];
  const int buckets = experts + 1;
  int* running = smem;                        // [buckets]
  int* warp_counts = smem + buckets;          // [8][buckets]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int b = threadIdx.x; b < buckets; b += blockDim.x) running[b] = starts[static_cast<int64_t>(blockIdx.x) * buckets + b];
  for (int b = threadIdx.x; b < 8 * buckets; b += blockDim.x) warp_counts[b] = 0;
  __syncthreads();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kRouteChunk;
  const int64_t end = min(base + kRouteChunk, n);
  for (int64_t round = base; round < end; round += kRouteThreads) {
    const int64_t i = round + threadIdx.x;
    const bool live = i < end;
    const int64_t id = live ? ids[i] : -1;
    const int b = live ? bucket_of(id, experts) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, b);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (live && rank == 0) warp_counts[warp * buckets + b] = __popc(peers);
    __syncthreads();
    if (live) {
      int pos = running[b] + rank;
      for (int w = 0; w < warp; ++w) pos += warp_counts[w * buckets + b];
      perm[pos] = i;
      if (ids_g) ids_g[pos] = (b == experts) ? static_cast<int64_t>(experts - 1) : id;
      if (inverse) inverse[i] = pos;
    }
    __syncthreads();
    for (int bb = threadIdx.x; bb < buckets; bb += blockDim.x) {
      int add = 0;
      for (int w = 0; w < 8; ++w) {
        add += warp_counts[w * buckets + bb];
        warp_counts[w * buckets + bb] = 0;
      }
      running[bb] += add;
    }
    __syncthreads();
  }
}

// The router of Transformers' MoE blocks (Qwen3MoeTopKRouter.forward: softmax in float32 over the experts, top-k,
// the k weights renormalised to sum to one) fused with the first pass of the routing sort: CTA c computes the tokens
// whose assignments t * top_k + j fall in chunk c (kRouteChunk assignments, the histogram's chunking) and counts the
// chunk's assignments per expert, so route_scan and route_scatter follow directly. One warp per token, the token's
// logits spread over the lanes (expert e at lane e % 32, slot e / 32); the maximum and the sum go through butterfly
// shuffles; the top k by k rounds of a warp arg-max (largest probability, the smaller expert index on a tie), so
// the k weights come out in descending order as torch.topk returns them. A token whose assignments straddle two
// chunks is computed by both CTAs, which write the same values.
constexpr int kRouterWarps = 16;

__device__ __forceinline__ float logit_value(const float* p, int64_t i) { return p[i]; }
__device__ __forceinline__ float logit_value(const __nv_bfloat16* p, int64_t i) { return __bfloat162float(p[i]); }

template <typename L, int PER>
__global__ void __launch_bounds__(kRouterWarps * 32) router_topk(const L* __restrict__ logits, int64_t tokens,
                                                                int experts, int top_k, bool norm,
                                                                float* __restrict__ probs,
                                                                int64_t* __restrict__ index,
                                                                float* __restrict__ weights, int* __restrict__ counts) {
  extern __shared__ int router_hist[];
  const int buckets = experts + 1;
  for (int b = threadIdx.x; b < buckets; b += blockDim.x) router_hist[b] = 0;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t a0 = static_cast<int64_t>(blockIdx.x) * kRouteChunk;
  const int64_t a1 = min(a0 + kRouteChunk, tokens * top_k);
  const int64_t t0 = a0 / top_k, t1 = (a1 + top_k - 1) / top_k;
  for (int64_t t = t0 + warp; t < t1; t += kRouterWarps) {
    const L* row = logits + t * experts;
    float v[PER];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = i * 32 + lane;
      v[i] = e < experts ? logit_value(row, e) : -INFINITY;
      m = fmaxf(m, v[i]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = i * 32 + lane;
      v[i] = e < experts ? expf(v[i] - m) : 0.f;
      sum += v[i];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = i * 32 + lane;
      v[i] = __fdiv_rn(v[i], sum);
      if (probs != nullptr && e < experts) probs[t * experts + e] = v[i];
    }
    uint32_t taken = 0;
    float mine_v = 0.f;
    int mine_i = 0;
    for (int j = 0; j < top_k; ++j) {
      float bv = -1.f;
      int bi = INT_MAX;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int e = i * 32 + lane;
        if (e < experts && !((taken >> i) & 1u) && v[i] > bv) bv = v[i], bi = e;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ov > bv || (ov == bv && oi < bi)) bv = ov, bi = oi;
      }
      if (bi != INT_MAX && (bi & 31) == lane) taken |= 1u << (bi >> 5);  // (NaN logits select nothing)
      if (lane == j) mine_v = bv, mine_i = bi;
    }
    float wsum = 0.f;
    for (int j = 0; j < top_k; ++j) wsum += __shfl_sync(0xffffffffu, mine_v, j);
    if (lane < top_k) {
      const int64_t a = t * top_k + lane;
      index[a] = mine_i;
      weights[a] = norm ? __fdiv_rn(mine_v, wsum) : mine_v;
      if (a >= a0 && a < a1) atomicAdd(&router_hist[mine_i < experts ? mine_i : experts], 1);
    }
  }
  __syncthreads();
  for (int b = threadIdx.x; b < buckets; b += blockDim.x)
    counts[static_cast<int64_t>(blockIdx.x) * buckets + b] = router_hist[b];
}

// selected[i] = hidden[perm[i] / top_k] (zero past the real rows); weights_g[i] = weights[perm[i]].
// One warp per row, 16-byte vectors.
template <typename W>
__global__ void __launch_bounds__(256) gather_rows(const uint4* __restrict__ hidden, int64_t vec_per_row,
                                                   int top_k, const int64_t* __restrict__ perm,
                                                   const int32_t* __restrict__ offsets, int experts, int64_t rows,
                                                   const W* __restrict__ weights, W* __restrict__ weights_g,
                                                   uint4* __restrict__ selected) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t valid = offsets[experts - 1];
  const int64_t src = perm[row];
  uint4* dst = selected + row * vec_per_row;
  if (weights_g != nullptr && lane == 0) weights_g[row] = weights[src];
  if (row < valid) {
    // eight 16-byte loads in flight per lane before their stores; the stores stream (the sorted copy is read once,
    // later, by the product) so that the token-major source stays in L2 for the other k - 1 reads of each row
    const uint4* s = hidden + (src / top_k) * vec_per_row;
    int64_t v = lane;
    for (; v + 7 * 32 < vec_per_row; v += 8 * 32) {
      uint4 q[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) q[i] = __ldg(s + v + 32 * i);
#pragma unroll
      for (int i = 0; i < 8; ++i) __stcs(dst + v + 32 * i, q[i]);
    }
    for (; v < vec_per_row; v += 32) __stcs(dst + v, __ldg(s + v));
  } else {
    for (int64_t v = lane; v < vec_per_row; v += 32) dst[v] = make_uint4(0, 0, 0, 0);
  }
}

__device__ __forceinline__ float weight_value(const float* w, int64_t i) { return w[i]; }
__device__ __forceinline__ float weight_value(const __nv_bfloat16* w, int64_t i) { return __bfloat162float(w[i]); }

// out[t] = bf16(sum_j y[r_j] * w_g[r_j]), r_j = inverse[t * top_k + j]. One CTA per token, 8 bf16 per thread
// and step. F32 weights: each product rounded to float32 (bf16 * f32 promotes), summed in float32. BF16 weights:
// each product rounded to bf16 (bf16 * bf16), summed in float32. No weights: a plain float32 sum. The token's row
// indices and weights are read once into shared memory, and every thread issues the loads of all its rows before
// it sums them (in order j = 0, 1, ...), so a token costs one round trip to memory rather than top_k.
// TOKEN_MAJOR (the combine): y holds the rows in token-major order, row t * top_k + j for the token's j-th
// assignment (the down product stored them there through the permutation), and weights_g is the routing weights
// in the same (tokens, top_k) order; inverse only tells which assignments are sentinels (never stored).
constexpr int kUnpermuteGroup = 8;  // rows whose loads are in flight together
template <typename W, bool TOKEN_MAJOR = false>
__global__ void __launch_bounds__(256) unpermute_rows(const uint4* __restrict__ y, const int64_t* __restrict__ inverse,
                                                     const W* __restrict__ weights_g,
                                                     const int32_t* __restrict__ offsets, int experts,
                                                     int top_k, int64_t vec_per_row, uint4* __restrict__ out) {
  extern __shared__ int64_t unpermute_smem[];  // the token's rows (-1: a sentinel), then their weights
  int64_t* rows_s = unpermute_smem;
  float* w_s = reinterpret_cast<float*>(unpermute_smem + top_k);
  const int64_t t = blockIdx.x;
  const int64_t valid = offsets[experts - 1];
  for (int j = threadIdx.x; j < top_k; j += blockDim.x) {
    const int64_t r = inverse[t * top_k + j];
    const int64_t src = TOKEN_MAJOR ? t * top_k + j : r;
    rows_s[j] = r < valid ? src : -1;  // a sentinel row: masked to zero (_moe.py:116)
    w_s[j] = (weights_g != nullptr && r < valid) ? weight_value(weights_g, src) : 1.f;
  }
  __syncthreads();
  const bool round_bf16 = sizeof(W) == 2;
  for (int64_t v = threadIdx.x; v < vec_per_row; v += blockDim.x) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j0 = 0; j0 < top_k; j0 += kUnpermuteGroup) {
      uint4 q[kUnpermuteGroup];
#pragma unroll
      for (int j = 0; j < kUnpermuteGroup; ++j) {
        const int64_t r = j0 + j < top_k ? rows_s[j0 + j] : -1;
        q[j] = r >= 0 ? __ldg(y + r * vec_per_row + v) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int j = 0; j < kUnpermuteGroup; ++j) {
        if (j0 + j >= top_k || rows_s[j0 + j] < 0) continue;
        const uint32_t words[4] = {q[j].x, q[j].y, q[j].z, q[j].w};
        if (weights_g == nullptr) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            acc[2 * e] = __fadd_rn(acc[2 * e], bf16_lo(words[e]));
            acc[2 * e + 1] = __fadd_rn(acc[2 * e + 1], bf16_hi(words[e]));
          }
        } else {
          const float w = w_s[j0 + j];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float p0 = __fmul_rn(bf16_lo(words[e]), w), p1 = __fmul_rn(bf16_hi(words[e]), w);
            if (round_bf16) {
              p0 = bf16_round(p0);
              p1 = bf16_round(p1);
            }
            acc[2 * e] = __fadd_rn(acc[2 * e], p0);
            acc[2 * e + 1] = __fadd_rn(acc[2 * e + 1], p1);
          }
        }
      }
    }
    out[t * vec_per_row + v] = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                                          pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
  }
}

// grad_y[i] = bf16(grad_out[tok] * w_g[i]); grad_weights[perm[i]] = sum_h grad_out[tok][h] * y[i][h]. One warp per
// routed row, eight rows per CTA, 16-byte vectors; the dot product reduced with shuffles.
template <typename W>
__global__ void __launch_bounds__(256) unpermute_backward_rows(const uint4* __restrict__ grad_out,
                                                               const uint4* __restrict__ y,
                                                               const int64_t* __restrict__ perm,
                                                               const W* __restrict__ weights_g,
                                                               const int32_t* __restrict__ offsets, int experts,
                                                               int top_k, int64_t rows, int64_t vec_per_row,
                                                               uint4* __restrict__ grad_y,
                                                               float* __restrict__ grad_weights) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (i >= rows) return;
  const int64_t valid = offsets[experts - 1];
  const int64_t src = perm[i];
  const bool live = i < valid;
  const float w = live ? weight_value(weights_g, i) : 0.f;
  const bool round_bf16 = sizeof(W) == 2;
  float dot = 0.f;
  const uint4* g_row = grad_out + (src / top_k) * vec_per_row;
  const uint4* y_row = y + i * vec_per_row;
  uint4* o_row = grad_y + i * vec_per_row;
  for (int64_t v = lane; v < vec_per_row; v += 32) {
    uint4 o = make_uint4(0, 0, 0, 0);
    if (live) {
      const uint4 g = __ldg(g_row + v);
      const uint4 q = __ldcs(y_row + v);  // read once: do not keep in L2
      const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
      const uint32_t yw[4] = {q.x, q.y, q.z, q.w};
      uint32_t ow[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float g0 = bf16_lo(gw[e]), g1 = bf16_hi(gw[e]);
        ow[e] = pack_bf16x2(__fmul_rn(g0, w), __fmul_rn(g1, w));
        if (round_bf16) {  // bf16 weights: autograd's sum of bf16 products
          dot = __fadd_rn(dot, bf16_round(__fmul_rn(g0, bf16_lo(yw[e]))));
          dot = __fadd_rn(dot, bf16_round(__fmul_rn(g1, bf16_hi(yw[e]))));
        } else {
          dot = fmaf(g0, bf16_lo(yw[e]), dot);
          dot = fmaf(g1, bf16_hi(yw[e]), dot);
        }
      }
      o = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    }
    o_row[v] = o;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
  if (lane == 0) grad_weights[src] = live ? dot : 0.f;
}

// The routing weights' gradient from the per-row partial dot products of the down stack's input-gradient product:
// grad_weights[perm[i]] = sum over b < blocks of parts[i * ld + b] (in order b = 0, 1, ...) for the experts' rows,
// zero for the sentinel rows (whose partials nobody writes). One thread per routed row.
__global__ void __launch_bounds__(256) weight_grad_rows(const float* __restrict__ parts, int64_t ld, int blocks,
                                                       const int64_t* __restrict__ perm, int64_t rows,
                                                       const int32_t* __restrict__ offsets, int experts,
                                                       float* __restrict__ grad_weights) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows) return;
  float acc = 0.f;
  if (i < offsets[experts - 1]) {
    const float* p = parts + i * ld;
    for (int b = 0; b < blocks; ++b) acc = __fadd_rn(acc, p[b]);
  }
  grad_weights[perm[i]] = acc;
}

// The tile map: tiles per expert, their running sum, and for every tile index t < max_tiles the expert (by binary
// search over the running sums; spares clamp to the last expert) and the first row.
__global__ void __launch_bounds__(1024) tile_map_kernel(const int32_t* __restrict__ offsets, int experts,
                                                        int block_m, int64_t max_tiles,
                                                        int32_t* __restrict__ tile_expert,
                                                        int32_t* __restrict__ tile_row, int32_t* __restrict__ tiles) {
  extern __shared__ int tm[];
  int* ends = tm;              // inclusive running tile count per expert
  int* starts = tm + experts;  // first row per expert
  __shared__ int warp_sums[32];
  // thread i takes a run of `per` experts; a block-wide scan of the runs' tile counts gives each run its start
  const int per = (experts + blockDim.x - 1) / blockDim.x;
  const int e0 = min(experts, static_cast<int>(threadIdx.x) * per), e1 = min(experts, e0 + per);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int local = 0;
  for (int e = e0; e < e1; ++e) local += (offsets[e] - (e > 0 ? offsets[e - 1] : 0) + block_m - 1) / block_m;
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int nw = (blockDim.x + 31) >> 5;
    int v = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += u;
    }
    if (lane < nw) warp_sums[lane] = v;  // inclusive over warps
  }
  __syncthreads();
  int run = (warp > 0 ? warp_sums[warp - 1] : 0) + incl - local;
  for (int e = e0; e < e1; ++e) {
    const int prev = e > 0 ? offsets[e - 1] : 0;
    starts[e] = prev;
    run += (offsets[e] - prev + block_m - 1) / block_m;
    ends[e] = run;
  }
  if (threadIdx.x == blockDim.x - 1) *tiles = run;  // the last run ends at the total
  __syncthreads();
  for (int64_t t = threadIdx.x; t < max_tiles; t += blockDim.x) {
    int lo = 0, hi = experts;  // first e with ends[e] > t
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (ends[mid] > t) hi = mid; else lo = mid + 1;
    }
    const int e = lo < experts ? lo : experts - 1;
    const int before = ends[e] - (ends[e] - (e > 0 ? ends[e - 1] : 0));
    tile_expert[t] = e;
    tile_row[t] = starts[e] + static_cast<int>(t - before) * block_m;
  }
}

}  // namespace meep2b

using namespace meep2b;

namespace meep2b {
// Per routed row i (expert order): the token it reads (perm[i] / top_k) and its routing weight as float32.
__global__ void routed_rows(const int64_t* __restrict__ perm, int64_t n, int top_k, const void* __restrict__ weights,
                            bool bf16, int32_t* __restrict__ token_rows, float* __restrict__ weights_g) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int64_t a = perm[i];
  token_rows[i] = static_cast<int32_t>(a / top_k);
  if (weights != nullptr && weights_g != nullptr)
    weights_g[i] = bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(weights)[a])
                        : static_cast<const float*>(weights)[a];
}
}  // namespace meep2b

extern "C" {

size_t meep2b_route_workspace_bytes(int64_t assignments, int32_t experts) {
  const int64_t blocks = (assignments + kRouteChunk - 1) / kRouteChunk;
  return static_cast<size_t>((blocks > 0 ? blocks : 1) * (experts + 1)) * sizeof(int);
}

int meep2b_route(const int64_t* expert_ids, int64_t assignments, int32_t experts, int64_t* perm,
                 int64_t* expert_ids_g, int32_t* offsets, int64_t* inverse, void* workspace,
                 size_t workspace_bytes, void* stream) {
  // positions and offsets are int32 in the kernels (as the reference's int32 offsets, _moe.py:84)
  if (experts < 1 || experts + 1 > kMaxBuckets || assignments < 0 || assignments > INT32_MAX)
    return MEEP2B_ERR_SHAPE;
  if (workspace_bytes < meep2b_route_workspace_bytes(assignments, experts)) return MEEP2B_ERR_SHAPE;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  if (assignments == 0) {
    cudaMemsetAsync(offsets, 0, sizeof(int32_t) * experts, s);
    return launch_status();
  }
  const int blocks = static_cast<int>((assignments + kRouteChunk - 1) / kRouteChunk);
  int* counts = static_cast<int*>(workspace);
  const size_t hist_smem = sizeof(int) * (experts + 1);
  route_histogram<<<blocks, kRouteThreads, hist_smem, s>>>(expert_ids, assignments, experts, counts);
  route_scan<<<1, 1024, 0, s>>>(counts, blocks, experts, offsets);
  const size_t scatter_smem = sizeof(int) * 9 * (experts + 1);
  route_scatter<<<blocks, kRouteThreads, scatter_smem, s>>>(expert_ids, assignments, experts, counts, perm,
                                                            expert_ids_g, inverse);
  return launch_status();
}

int meep2b_route_logits(const void* logits, int32_t logits_dtype, int64_t tokens, int32_t experts, int32_t top_k,
                        int32_t norm_topk_prob, float* probs, int64_t* top_k_index, float* top_k_weights,
                        int64_t* perm, int64_t* expert_ids_g, int32_t* offsets, int64_t* inverse, void* workspace,
                        size_t workspace_bytes, void* stream) {
  if (experts < 1 || experts + 1 > kMaxBuckets || tokens < 0 || top_k < 1 || top_k > 32 || top_k > experts)
    return MEEP2B_ERR_SHAPE;
  if (tokens > INT32_MAX / top_k) return MEEP2B_ERR_SHAPE;
  if (logits_dtype != MEEP2B_F32 && logits_dtype != MEEP2B_BF16) return MEEP2B_ERR_DTYPE;
  const int64_t assignments = tokens * top_k;
  if (workspace_bytes < meep2b_route_workspace_bytes(assignments, experts)) return MEEP2B_ERR_SHAPE;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  if (assignments == 0) {
    cudaMemsetAsync(offsets, 0, sizeof(int32_t) * experts, s);
    return launch_status();
  }
  const int blocks = static_cast<int>((assignments + kRouteChunk - 1) / kRouteChunk);
  int* counts = static_cast<int*>(workspace);
  const size_t hist_smem = sizeof(int) * (experts + 1);
  const int per = (experts + 31) / 32;
  const bool norm = norm_topk_prob != 0;
#define MEEP2B_ROUTER(L, PER)                                                                               \
  router_topk<L, PER><<<blocks, kRouterWarps * 32, hist_smem, s>>>(static_cast<const L*>(logits), tokens, experts, \
                                                                  top_k, norm, probs, top_k_index, top_k_weights,  \
                                                                  counts)
#define MEEP2B_ROUTER_PER(L)          \
  if (per <= 1) MEEP2B_ROUTER(L, 1);  \
  else if (per <= 2) MEEP2B_ROUTER(L, 2); \
  else if (per <= 4) MEEP2B_ROUTER(L, 4); \
  else if (per <= 8) MEEP2B_ROUTER(L, 8); \
  else if (per <= 16) MEEP2B_ROUTER(L, 16); \
  else MEEP2B_ROUTER(L, 32);
  if (logits_dtype == MEEP2B_BF16) {
    MEEP2B_ROUTER_PER(__nv_bfloat16)
  } else {
    MEEP2B_ROUTER_PER(float)
  }
#undef MEEP2B_ROUTER_PER
#undef MEEP2B_ROUTER
  route_scan<<<1, 1024, 0, s>>>(counts, blocks, experts, offsets);
  const size_t scatter_smem = sizeof(int) * 9 * (experts + 1);
  route_scatter<<<blocks, kRouteThreads, scatter_smem, s>>>(top_k_index, assignments, experts, counts, perm,
                                                            expert_ids_g, inverse);
  return launch_status();
}

int meep2b_routed_rows(const int64_t* perm, int64_t assignments, int32_t top_k, const void* weights,
                       int32_t weights_dtype, int32_t* token_rows, float* weights_g, void* stream) {
  if (top_k < 1 || assignments < 0) return MEEP2B_ERR_SHAPE;
  if (weights != nullptr && weights_dtype != MEEP2B_F32 && weights_dtype != MEEP2B_BF16) return MEEP2B_ERR_DTYPE;
  if (assignments / top_k > INT32_MAX) return MEEP2B_ERR_SHAPE;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  if (assignments == 0) return MEEP2B_OK;
  const unsigned grid = static_cast<unsigned>((assignments + 255) / 256);
  routed_rows<<<grid, 256, 0, s>>>(perm, assignments, top_k, weights, weights_dtype == MEEP2B_BF16, token_rows,
                                   weights_g);
  return launch_status();
}

int meep2b_gather(const void* hidden, int64_t tokens, int64_t hidden_dim, int32_t top_k, const int64_t* perm,
                  const int32_t* offsets, int32_t experts, const void* weights, int32_t weights_dtype,
                  void* weights_g, void* selected, void* stream) {
  if (top_k < 1 || experts < 1 || tokens < 0 || hidden_dim % 8 != 0) return MEEP2B_ERR_SHAPE;
  if (!aligned16(hidden) || !aligned16(selected)) return MEEP2B_ERR_ALIGN;
  if ((weights_g != nullptr) && weights_dtype != MEEP2B_F32 && weights_dtype != MEEP2B_BF16) return MEEP2B_ERR_DTYPE;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  const int64_t rows = tokens * top_k;
  if (rows == 0) return MEEP2B_OK;
  const int64_t vec = hidden_dim / 8;
  const unsigned grid = static_cast<unsigned>((rows + 7) / 8);
  if (weights_dtype == MEEP2B_BF16)
    gather_rows<__nv_bfloat16><<<grid, 256, 0, s>>>(
        static_cast<const uint4*>(hidden), vec, top_k, perm, offsets, experts, rows,
        static_cast<const __nv_bfloat16*>(weights), static_cast<__nv_bfloat16*>(weights_g),
        static_cast<uint4*>(selected));
  else
    gather_rows<float><<<grid, 256, 0, s>>>(static_cast<const uint4*>(hidden), vec, top_k, perm, offsets, experts,
                                            rows, static_cast<const float*>(weights), static_cast<float*>(weights_g),
                                            static_cast<uint4*>(selected));
  return launch_status();
}

int meep2b_unpermute(const void* y, const int64_t* inverse, const void* weights_g, int32_t weights_dtype,
                     const int32_t* offsets, int32_t experts, int64_t tokens, int32_t top_k, int64_t hidden_dim,
                     void* out, void* stream) {
  if (top_k < 1 || experts < 1 || tokens < 0 || hidden_dim % 8 != 0) return MEEP2B_ERR_SHAPE;
  if (!aligned16(y) || !aligned16(out)) return MEEP2B_ERR_ALIGN;
  if (weights_g != nullptr && weights_dtype != MEEP2B_F32 && weights_dtype != MEEP2B_BF16) return MEEP2B_ERR_DTYPE;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  if (tokens == 0) return MEEP2B_OK;
  const int64_t vec = hidden_dim / 8;
  const int threads = vec >= 256 ? 256 : static_cast<int>(((vec + 31) / 32) * 32);
  const size_t smem = static_cast<size_t>(top_k) * (sizeof(int64_t) + sizeof(float));
  if (smem > 48 * 1024) return MEEP2B_ERR_SHAPE;
  if (weights_g != nullptr && weights_dtype == MEEP2B_BF16)
    unpermute_rows<__nv_bfloat16><<<static_cast<unsigned>(tokens), threads, smem, s>>>(
        static_cast<const uint4*>(y), inverse, static_cast<const __nv_bfloat16*>(weights_g), offsets, experts, top_k,
        vec, static_cast<uint4*>(out));
  else
    unpermute_rows<float><<<static_cast<unsigned>(tokens), threads, smem, s>>>(
        static_cast<const uint4*>(y), inverse, static_cast<const float*>(weights_g), offsets, experts, top_k, vec,
        static_cast<uint4*>(out));
  return launch_status();
}

int meep2b_combine(const void* y_tok, const int64_t* inverse, const void* weights, int32_t weights_dtype,
                   const int32_t* offsets, int32_t experts, int64_t tokens, int32_t top_k, int64_t hidden_dim,
                   void* out, void* stream) {
  if (top_k < 1 || experts < 1 || tokens < 0 || hidden_dim % 8 != 0) return MEEP2B_ERR_SHAPE;
  if (!aligned16(y_tok) || !aligned16(out)) return MEEP2B_ERR_ALIGN;
  if (weights != nullptr && weights_dtype != MEEP2B_F32 && weights_dtype != MEEP2B_BF16) return MEEP2B_ERR_DTYPE;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  if (tokens == 0) return MEEP2B_OK;
  const int64_t vec = hidden_dim / 8;
  const int threads = vec >= 256 ? 256 : static_cast<int>(((vec + 31) / 32) * 32);
  const size_t smem = static_cast<size_t>(top_k) * (sizeof(int64_t) + sizeof(float));
  if (smem > 48 * 1024) return MEEP2B_ERR_SHAPE;
  if (weights != nullptr && weights_dtype == MEEP2B_BF16)
    unpermute_rows<__nv_bfloat16, true><<<static_cast<unsigned>(tokens), threads, smem, s>>>(
        static_cast<const uint4*>(y_tok), inverse, static_cast<const __nv_bfloat16*>(weights), offsets, experts,
        top_k, vec, static_cast<uint4*>(out));
  else
    unpermute_rows<float, true><<<static_cast<unsigned>(tokens), threads, smem, s>>>(
        static_cast<const uint4*>(y_tok), inverse, static_cast<const float*>(weights), offsets, experts, top_k, vec,
        static_cast<uint4*>(out));
  return launch_status();
}

int meep2b_unpermute_backward(const void* grad_out, const void* y, const int64_t* perm, const void* weights_g,
                              int32_t weights_dtype, const int32_t* offsets, int32_t experts, int64_t assignments,
                              int32_t top_k, int64_t hidden_dim, void* grad_y, float* grad_weights, void* stream) {
  if (top_k < 1 || experts < 1 || assignments < 0 || hidden_dim % 8 != 0) return MEEP2B_ERR_SHAPE;
  if (!aligned16(grad_out) || !aligned16(y) || !aligned16(grad_y)) return MEEP2B_ERR_ALIGN;
  if (weights_dtype != MEEP2B_F32 && weights_dtype != MEEP2B_BF16) return MEEP2B_ERR_DTYPE;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  if (assignments == 0) return MEEP2B_OK;
  const int64_t vec = hidden_dim / 8;
  if (weights_dtype == MEEP2B_BF16)
    unpermute_backward_rows<__nv_bfloat16><<<static_cast<unsigned>((assignments + 7) / 8), 256, 0, s>>>(
        static_cast<const uint4*>(grad_out), static_cast<const uint4*>(y), perm,
        static_cast<const __nv_bfloat16*>(weights_g), offsets, experts, top_k, assignments, vec,
        static_cast<uint4*>(grad_y), grad_weights);
  else
    unpermute_backward_rows<float><<<static_cast<unsigned>((assignments + 7) / 8), 256, 0, s>>>(
        static_cast<const uint4*>(grad_out), static_cast<const uint4*>(y), perm, static_cast<const float*>(weights_g),
        offsets, experts, top_k, assignments, vec, static_cast<uint4*>(grad_y), grad_weights);
  return launch_status();
}

int meep2b_weight_grad(const float* parts, int64_t ld, int32_t blocks, const int64_t* perm, int64_t assignments,
                       const int32_t* offsets, int32_t experts, float* grad_weights, void* stream) {
  if (experts < 1 || assignments < 0 || blocks < 0 || ld < blocks) return MEEP2B_ERR_SHAPE;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  if (assignments == 0) return MEEP2B_OK;
  weight_grad_rows<<<static_cast<unsigned>((assignments + 255) / 256), 256, 0, s>>>(parts, ld, blocks, perm,
                                                                                   assignments, offsets, experts,
                                                                                   grad_weights);
  return launch_status();
}

int meep2b_tile_map(const int32_t* offsets, int32_t experts, int64_t rows, int32_t block_m, int32_t* tile_expert,
                    int32_t* tile_row, int32_t* tiles, void* stream) {
  if (experts < 1 || rows < 0 || block_m < 1 || experts > 16384) return MEEP2B_ERR_SHAPE;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  const int64_t max_tiles = rows / block_m + experts;
  const int smem = static_cast<int>(sizeof(int)) * 2 * experts;  // up to 128 KB at 16384 experts
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(tile_map_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
    cudaGetLastError();
    return MEEP2B_ERR_LAUNCH;
  }
  tile_map_kernel<<<1, 1024, smem, s>>>(offsets, experts, block_m, max_tiles, tile_expert, tile_row, tiles);
  return launch_status();
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------------------------
// Routing without allocation.
//
// meep2b_route takes its bucket-count table as a caller-provided workspace. Some callers cannot provide one: a
// host runtime that hands this library only the input and output buffers it owns and has no device allocator to
// lend (an FFI caller outside PyTorch, a serving process whose device memory is reserved up front), or code that
// must not call cudaMalloc because it would synchronise the device or break a memory budget. For them,
// meep2b_route_noalloc keeps that table in a fixed array in device memory that this library declares at file
// scope, so the call allocates nothing. The array lives on every GPU that loads the library until the process
// exits. Its host-side name is only a stand-in for the symbol: the device address comes from cudaGetSymbolAddress
// (which allocates nothing), looked up again on each call made outside a stream capture, so that it stays right
// after a cudaDeviceReset (the module is loaded anew and the array may move); a call on a stream being captured
// uses the address of the last lookup on that device.
namespace meep2b {

constexpr int64_t kNoAllocRouteWords = 65536;  // 256 KB of int32 bucket counts
static __device__ __align__(256) int g_route_scratch[kNoAllocRouteWords];

constexpr int kMaxDevices = 64;
static int* g_route_scratch_addr[kMaxDevices] = {nullptr};
static std::mutex g_route_scratch_mutex;

// The device address of g_route_scratch on the current device (the stream's, made current by bind_stream_device):
// looked up with that device current unless the stream is being captured and an earlier lookup exists.
static int route_scratch_address(cudaStream_t stream, int** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return MEEP2B_ERR_LAUNCH;
  }
  if (dev < 0 || dev >= kMaxDevices) return MEEP2B_ERR_DEVICE;
  cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &capturing) != cudaSuccess) {
    cudaGetLastError();
    return MEEP2B_ERR_LAUNCH;
  }
  std::lock_guard<std::mutex> lock(g_route_scratch_mutex);
  if (capturing == cudaStreamCaptureStatusNone || g_route_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_route_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return MEEP2B_ERR_LAUNCH;
    }
    g_route_scratch_addr[dev] = static_cast<int*>(p);
  }
  *out = g_route_scratch_addr[dev];
  return MEEP2B_OK;
}

}  // namespace meep2b

extern "C" int meep2b_route_noalloc(const int64_t* expert_ids, int64_t assignments, int32_t experts, int64_t* perm,
                                    int64_t* expert_ids_g, int32_t* offsets, int64_t* inverse, void* stream) {
  using namespace meep2b;
  if (experts < 1 || experts + 1 > kMaxBuckets || assignments < 0) return MEEP2B_ERR_SHAPE;
  const int64_t blocks = (assignments + kRouteChunk - 1) / kRouteChunk;
  if (blocks * (experts + 1) > kNoAllocRouteWords) return MEEP2B_ERR_SHAPE;  // beyond the fixed table
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  int* counts = nullptr;
  MEEP2B_TRY(route_scratch_address(s, &counts));
  if (assignments == 0) {
    cudaMemsetAsync(offsets, 0, sizeof(int32_t) * experts, s);
    return launch_status();
  }
  // Every entry of the table this call reads is first written by route_histogram, so nothing left over from an
  // earlier call leaks in; nothing needs clearing.
  const size_t hist_smem = sizeof(int) * (experts + 1);
  route_histogram<<<static_cast<int>(blocks), kRouteThreads, hist_smem, s>>>(expert_ids, assignments, experts,
                                                                            counts);
  route_scan<<<1, 1024, 0, s>>>(counts, static_cast<int>(blocks), experts, offsets);
  const size_t scatter_smem = sizeof(int) * 9 * (experts + 1);
  route_scatter<<<static_cast<int>(blocks), kRouteThreads, scatter_smem, s>>>(expert_ids, assignments, experts,
                                                                              counts, perm, expert_ids_g, inverse);
  return launch_status();
}

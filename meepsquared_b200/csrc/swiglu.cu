// The SwiGLU gate between the two grouped products when the layer runs unfused (FP8 tensor-core products, adapters
// of rank above 16): Transformers' _default_apply_gate, which the reference calls as experts._apply_gate
// (_moe.py:119): gate, up = gate_up.chunk(2, -1); h = silu(gate) * up. Same arithmetic as the fused products'
// SwiGLU and dSwiGLU epilogues (grouped_gemm.cu): h = bf16(bf16(silu(g)) * u); backward dact = bf16(dh * u),
// d_up = dh * bf16(silu(g)), d_gate = dact * sig(g) * (1 + g (1 - sig(g))). HBM bound: eight columns a thread,
// 16-byte loads and stores.

namespace meep2b {
namespace swiglu {

__global__ void __launch_bounds__(256) swiglu_rows(const uint4* __restrict__ gate_up, int64_t rows, int64_t vec,
                                                   uint4* __restrict__ h) {
  const int64_t n = rows * vec;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / vec, c = i - r * vec;
    const uint4 g = __ldcs(gate_up + r * 2 * vec + c);
    const uint4 u = __ldcs(gate_up + r * 2 * vec + vec + c);
    const uint32_t gw[4] = {g.x, g.y, g.z, g.w}, uw[4] = {u.x, u.y, u.z, u.w};
    uint32_t hw[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a0 = bf16_round(gemm::silu_f(bf16_lo(gw[j]))), a1 = bf16_round(gemm::silu_f(bf16_hi(gw[j])));
      hw[j] = pack_bf16x2(a0 * bf16_lo(uw[j]), a1 * bf16_hi(uw[j]));
    }
    h[i] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
  }
}

__global__ void __launch_bounds__(256) swiglu_backward_rows(const uint4* __restrict__ gate_up,
                                                            const uint4* __restrict__ grad_h, int64_t rows,
                                                            int64_t vec, uint4* __restrict__ grad_gate_up) {
  const int64_t n = rows * vec;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / vec, c = i - r * vec;
    const uint4 g = __ldcs(gate_up + r * 2 * vec + c);
    const uint4 u = __ldcs(gate_up + r * 2 * vec + vec + c);
    const uint4 d = __ldcs(grad_h + i);
    const uint32_t gw[4] = {g.x, g.y, g.z, g.w}, uw[4] = {u.x, u.y, u.z, u.w}, dw[4] = {d.x, d.y, d.z, d.w};
    uint32_t dgw[4], duw[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float dg[2], du[2];
#pragma unroll
      for (int hl = 0; hl < 2; ++hl) {
        const float gb = hl ? bf16_hi(gw[j]) : bf16_lo(gw[j]);
        const float ub = hl ? bf16_hi(uw[j]) : bf16_lo(uw[j]);
        const float dh = hl ? bf16_hi(dw[j]) : bf16_lo(dw[j]);
        const float act = bf16_round(gemm::silu_f(gb));  // the forward's activation, bit for bit
        const float sig = gemm::sigmoid_f(gb);
        const float dact = bf16_round(dh * ub);
        du[hl] = dh * act;
        dg[hl] = dact * sig * (1.0f + gb * (1.0f - sig));
      }
      dgw[j] = pack_bf16x2(dg[0], dg[1]);
      duw[j] = pack_bf16x2(du[0], du[1]);
    }
    grad_gate_up[r * 2 * vec + c] = make_uint4(dgw[0], dgw[1], dgw[2], dgw[3]);
    grad_gate_up[r * 2 * vec + vec + c] = make_uint4(duw[0], duw[1], duw[2], duw[3]);
  }
}

static int grid_for(int64_t n) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks = (n + 255) / 256;
  return static_cast<int>(blocks < int64_t(sms) * 8 ? (blocks > 0 ? blocks : 1) : int64_t(sms) * 8);
}

}  // namespace swiglu
}  // namespace meep2b

extern "C" int meep2b_swiglu(const void* gate_up, int64_t rows, int64_t inter, void* h, void* stream) {
  using namespace meep2b;
  if (rows < 0 || inter < 1) return MEEP2B_ERR_SHAPE;
  if (inter % 8 || !aligned16(gate_up) || !aligned16(h)) return MEEP2B_ERR_ALIGN;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  if (rows == 0) return MEEP2B_OK;
  const int64_t vec = inter / 8;
  swiglu::swiglu_rows<<<swiglu::grid_for(rows * vec), 256, 0, s>>>(static_cast<const uint4*>(gate_up), rows, vec,
                                                                   static_cast<uint4*>(h));
  return launch_status();
}

extern "C" int meep2b_swiglu_backward(const void* gate_up, const void* grad_h, int64_t rows, int64_t inter,
                                      void* grad_gate_up, void* stream) {
  using namespace meep2b;
  if (rows < 0 || inter < 1) return MEEP2B_ERR_SHAPE;
  if (inter % 8 || !aligned16(gate_up) || !aligned16(grad_h) || !aligned16(grad_gate_up)) return MEEP2B_ERR_ALIGN;
  cudaStream_t s = as_stream(stream);
  MEEP2B_TRY(bind_stream_device(s));
  if (rows == 0) return MEEP2B_OK;
  const int64_t vec = inter / 8;
  swiglu::swiglu_backward_rows<<<swiglu::grid_for(rows * vec), 256, 0, s>>>(
      static_cast<const uint4*>(gate_up), static_cast<const uint4*>(grad_h), rows, vec,
      static_cast<uint4*>(grad_gate_up));
  return launch_status();
}

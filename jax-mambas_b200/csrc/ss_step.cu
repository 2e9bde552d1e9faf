// One recurrent decode step of the selective scan for sm_100a.
//
// The state update of S6.step / Mamba.step (mamba/mamba1.py:200-214), which
// the reference evaluates in JAX: for one new token per sequence,
//   delta_eff = softplus(delta + bias)             (if delta_softplus)
//   h <- exp(delta_eff A) h + delta_eff B u        (Euler; ZOH: expm1(.)/A B u)
//   out = (C . h + D u) * silu(z)
// with the state h (batch, dim, dstate) fp32 updated in place. The step moves
// a few bytes per state element and does one exponential each, so it is
// bound by HBM: each thread owns four states of one (batch, channel) row and
// streams them with 16-byte loads and stores; B and C rows are shared by the
// channels of a batch and come from L1.
#include "ss_common.cuh"
#include "ss_launch.h"

namespace mss {

// kTPC threads share a channel, each owning 4 consecutive states (16 bytes of
// the state row), so a warp streams whole 128-byte lines; the partial C . h
// sums are combined with xor-shuffles inside the thread group.
template <int NS>
struct StepCfg {
  static constexpr int kSPT = NS < 4 ? NS : 4;  // states per thread
  static constexpr int kTPC = NS / kSPT;        // threads per channel
};

template <int NS, typename T, bool kZOH>
__global__ void __launch_bounds__(128) ss_step_kernel(const StepParams p) {
  using Cfg = StepCfg<NS>;
  constexpr int kSPT = Cfg::kSPT, kTPC = Cfg::kTPC;
  const int gt = blockIdx.x * blockDim.x + threadIdx.x;
  const int d = gt / kTPC;
  const int part = gt % kTPC;
  const int b = blockIdx.y;
  const bool live = d < p.dim;
  const int dc = live ? d : 0;
  const size_t row = static_cast<size_t>(b) * p.dim + dc;
  float x = Elem<T>::ld(static_cast<const T*>(p.delta) + row);
  if (p.delta_bias) x += __ldg(p.delta_bias + dc);
  const float dl = p.delta_softplus ? softplus_f(x) : x;
  const float uv = Elem<T>::ld(static_cast<const T*>(p.u) + row);
  const T* Bb = static_cast<const T*>(p.B) + static_cast<size_t>(b) * NS;
  const T* Cb = static_cast<const T*>(p.C) + static_cast<size_t>(b) * NS;
  float* h = p.state + row * NS + part * kSPT;
  float hv[kSPT];
  if constexpr (kSPT == 4) {
    const float4 q = *reinterpret_cast<const float4*>(h);
    hv[0] = q.x; hv[1] = q.y; hv[2] = q.z; hv[3] = q.w;
  } else {
#pragma unroll
    for (int e = 0; e < kSPT; ++e) hv[e] = h[e];
  }
  float y = 0.f;
#pragma unroll
  for (int e = 0; e < kSPT; ++e) {
    const int n = part * kSPT + e;
    const float An = __ldg(p.A + dc * NS + n);
    const float ab = ex2(dl * An * kLog2e);
    const float bb = kZOH ? expm1f(dl * An) / An : dl;
    hv[e] = fmaf(ab, hv[e], bb * Elem<T>::ld(Bb + n) * uv);
    y = fmaf(Elem<T>::ld(Cb + n), hv[e], y);
  }
  if (live) {
    if constexpr (kSPT == 4) {
      *reinterpret_cast<float4*>(h) = make_float4(hv[0], hv[1], hv[2], hv[3]);
    } else {
#pragma unroll
      for (int e = 0; e < kSPT; ++e) h[e] = hv[e];
    }
  }
#pragma unroll
  for (int s = 1; s < kTPC; s <<= 1) y += __shfl_xor_sync(0xffffffffu, y, s);
  if (live && part == 0) {
    if (p.D) y = fmaf(__ldg(p.D + dc), uv, y);
    if (p.z) y *= silu_f(Elem<T>::ld(static_cast<const T*>(p.z) + row));
    Elem<T>::st(static_cast<T*>(p.out) + row, y);
  }
}

template <int NS, typename T, bool kZOH>
static cudaError_t launch_step_t(const StepParams& p, cudaStream_t stream) {
  const int threads = p.dim * StepCfg<NS>::kTPC;
  dim3 grid((threads + 127) / 128, p.batch);
  ss_step_kernel<NS, T, kZOH><<<grid, 128, 0, stream>>>(p);
  return cudaPeekAtLastError();
}

template <typename T, bool kZOH>
static cudaError_t launch_step_n(const StepParams& p, int dstate, cudaStream_t stream) {
  switch (dstate) {
    case 1: return launch_step_t<1, T, kZOH>(p, stream);
    case 2: return launch_step_t<2, T, kZOH>(p, stream);
    case 4: return launch_step_t<4, T, kZOH>(p, stream);
    case 8: return launch_step_t<8, T, kZOH>(p, stream);
    case 16: return launch_step_t<16, T, kZOH>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_step(const StepParams& p, int dstate, int io_dtype, int zoh,
                        cudaStream_t stream) {
  if (io_dtype == MSS_BF16)
    return zoh ? launch_step_n<__nv_bfloat16, true>(p, dstate, stream)
               : launch_step_n<__nv_bfloat16, false>(p, dstate, stream);
  return zoh ? launch_step_n<float, true>(p, dstate, stream)
             : launch_step_n<float, false>(p, dstate, stream);
}

}  // namespace mss

// Forward selective scan for sm_100a.
//
// Replaces SelectiveScanFwdKernel (native/selective_scan_cuda.cu:205-332) and
// folds in the caller-side math of S6.__call__/Mamba.__call__
// (mamba/mamba1.py:162-198, 308, 332): softplus(delta + bias) before the scan,
// the D skip and the silu(z) gate after it.
//
// One warp per (batch, channel) row; a CTA holds kFwdWarps channels of one
// batch so B/C runs are fetched once into L1 and reused by every warp.
#include "ss_common.cuh"
#include "ss_launch.h"

namespace mss {

constexpr int kFwdWarps = 4;

template <int NS, typename T, bool kZOH>
__global__ void __launch_bounds__(kFwdWarps * 32)
    ss_fwd_kernel(const FwdParams p) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int d = blockIdx.x * kFwdWarps + warp;
  const int b = blockIdx.y;
  if (d >= p.dim) return;  // the forward has no CTA-wide barrier

  const int L = p.seqlen;
  const size_t row = static_cast<size_t>(b) * p.dim + d;
  const T* u_row = static_cast<const T*>(p.u) + row * L;
  const T* dl_row = static_cast<const T*>(p.delta) + row * L;
  const T* z_row = p.z ? static_cast<const T*>(p.z) + row * L : nullptr;
  T* out_row = static_cast<T*>(p.out) + row * L;
  const T* B_b = static_cast<const T*>(p.B) + static_cast<size_t>(b) * NS * L;
  const T* C_b = static_cast<const T*>(p.C) + static_cast<size_t>(b) * NS * L;

  int len = L;
  if (p.seq_lens) len = max(0, min(L, p.seq_lens[b]));
  const float Dv = p.D ? __ldg(p.D + d) : 0.f;
  const float bias = p.delta_bias ? __ldg(p.delta_bias + d) : 0.f;

  float a2[NS];   // A * log2(e), so exp(delta*A) = 2^(delta*a2)
  float Av[NS];   // A itself (ZOH only)
  float carry[NS];
#pragma unroll
  for (int n = 0; n < NS; ++n) {
    Av[n] = __ldg(p.A + d * NS + n);
    a2[n] = Av[n] * kLog2e;
    carry[n] = p.h0 ? __ldg(p.h0 + row * NS + n) : 0.f;
  }

  for (int c = 0; c < p.n_chunks; ++c) {
    const int t0 = c * kChunk;
    const int tl = t0 + lane * kItems;
    float* cs = p.chunk_states + (row * p.n_chunks + c) * NS;

    if (t0 >= len) {
      // Whole chunk is padding (or past L): the state passes through.
      float zero[kItems];
#pragma unroll
      for (int k = 0; k < kItems; ++k) zero[k] = 0.f;
      store_run(out_row, tl, L, zero);
      if (lane == 0) {
#pragma unroll
        for (int n = 0; n < NS; ++n) cs[n] = carry[n];
      }
      continue;
    }

    float uv[kItems], dl[kItems], du[kItems], y[kItems];
    load_run(u_row, tl, len, uv);
    load_run(dl_row, tl, len, dl);
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      float v = dl[k] + bias;
      if (p.delta_softplus) v = softplus(v);
      dl[k] = (tl + k < len) ? v : 0.f;  // padding: delta = 0, so a = 1, b = 0
      du[k] = dl[k] * uv[k];
      y[k] = 0.f;
    }

#pragma unroll
    for (int n = 0; n < NS; ++n) {
      float Bv[kItems], Cv[kItems];
      load_run(B_b + static_cast<size_t>(n) * L, tl, len, Bv);
      load_run(C_b + static_cast<size_t>(n) * L, tl, len, Cv);
      float ab[kItems], bu[kItems];
      float P = 1.f, H = 0.f;
#pragma unroll
      for (int k = 0; k < kItems; ++k) {
        ab[k] = ex2(dl[k] * a2[n]);
        if constexpr (kZOH) {
          // b_bar = expm1(delta*A) / A * B   (mamba/selective_scan_cuda.py:77)
          bu[k] = Bv[k] * (expm1f(dl[k] * Av[n]) * (1.f / Av[n])) * uv[k];
        } else {
          bu[k] = Bv[k] * du[k];
        }
        H = fmaf(ab[k], H, bu[k]);
        P *= ab[k];
      }
      warp_scan_fwd(P, H, lane);
      float Pe = __shfl_up_sync(0xffffffffu, P, 1);
      float He = __shfl_up_sync(0xffffffffu, H, 1);
      const float Pt = __shfl_sync(0xffffffffu, P, 31);
      const float Ht = __shfl_sync(0xffffffffu, H, 31);
      if (lane == 0) {
        Pe = 1.f;
        He = 0.f;
      }
      float h = fmaf(Pe, carry[n], He);
#pragma unroll
      for (int k = 0; k < kItems; ++k) {
        h = fmaf(ab[k], h, bu[k]);
        y[k] = fmaf(Cv[k], h, y[k]);
      }
      carry[n] = fmaf(Pt, carry[n], Ht);
    }

    if (lane == 0) {
#pragma unroll
      for (int n = 0; n < NS; ++n) cs[n] = carry[n];
    }

    float zv[kItems];
    if (z_row) load_run(z_row, tl, len, zv);
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      float o = fmaf(Dv, uv[k], y[k]);
      if (z_row) o *= zv[k] * sigmoid(zv[k]);
      y[k] = (tl + k < len) ? o : 0.f;
    }
    store_run(out_row, tl, L, y);
  }

  if (p.last_state && lane == 0) {
#pragma unroll
    for (int n = 0; n < NS; ++n) p.last_state[row * NS + n] = carry[n];
  }
}

template <int NS, typename T, bool kZOH>
static cudaError_t launch_fwd_t(const FwdParams& p, cudaStream_t stream) {
  dim3 grid((p.dim + kFwdWarps - 1) / kFwdWarps, p.batch);
  ss_fwd_kernel<NS, T, kZOH><<<grid, kFwdWarps * 32, 0, stream>>>(p);
  return cudaPeekAtLastError();
}

template <typename T, bool kZOH>
static cudaError_t launch_fwd_n(const FwdParams& p, int dstate,
                                cudaStream_t stream) {
  switch (dstate) {
    case 1: return launch_fwd_t<1, T, kZOH>(p, stream);
    case 2: return launch_fwd_t<2, T, kZOH>(p, stream);
    case 4: return launch_fwd_t<4, T, kZOH>(p, stream);
    case 8: return launch_fwd_t<8, T, kZOH>(p, stream);
    case 16: return launch_fwd_t<16, T, kZOH>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_fwd(const FwdParams& p, int dstate, int io_dtype, int zoh,
                       cudaStream_t stream) {
  if (io_dtype == MSS_BF16) {
    return zoh ? launch_fwd_n<__nv_bfloat16, true>(p, dstate, stream)
               : launch_fwd_n<__nv_bfloat16, false>(p, dstate, stream);
  }
  return zoh ? launch_fwd_n<float, true>(p, dstate, stream)
             : launch_fwd_n<float, false>(p, dstate, stream);
}

}  // namespace mss

// Forward selective scan for sm_100a.
//
// Replaces SelectiveScanFwdKernel (native/selective_scan_cuda.cu:205-332) and
// folds in the caller-side math of S6.__call__/Mamba.__call__
// (mamba/mamba1.py:162-198, 308, 332): softplus(delta + bias) before the scan,
// the D skip and the silu(z) gate after it.
//
// Decomposition: the recurrence runs sequentially in time inside each lane,
// with no cross-lane scan. A lane owns kS states of one channel; kLPC = NS/kS
// lanes cover a channel, so a warp holds 32/kLPC channels and a CTA holds
// kCh = 32 channels of one batch. The CTA walks L in tiles of kTile steps,
// double-buffered:
//   0. TMA: one thread issues 1-D bulk copies of the tile's rows of delta, u,
//      z (per channel) and B, C (per state) into a staging buffer, completing
//      on an mbarrier; the next tile's copies fly while this tile computes;
//   1. transform: delta_eff = softplus(delta + bias), delta_eff*u and D*u are
//      formed once per element into fp32 work tiles, B and C are widened;
//   2. scan: each lane steps through the tile; per step and state one
//      2^(delta*A*log2 e) on the SFU and packed fp32x2 multiply-adds, then the
//      kS-state partial sums of C_t h_t are reduced over the channel's lanes;
//   3. emit: out = (y + D u) * silu(z) and the pre-gate y + D u (read by the
//      backward for dz) are written coalesced.
// The state at every MSS_CHUNK boundary is saved for the backward. Rows whose
// length or base address is not 16-byte aligned take the same path with the
// staging done by plain loads instead of TMA.
#include "ss_common.cuh"
#include "ss_launch.h"

namespace mss {

__device__ unsigned int g_fwd_device_error = 0;

constexpr int kCh = 32;    // channels per CTA
constexpr int kTile = 64;  // steps staged per pass
constexpr int kPad = 4;    // row padding (floats) of the fp32 work tiles
constexpr int kRow = kTile + kPad;
static_assert(kChunk % kTile == 0, "a carry checkpoint must end a tile");

template <int NS>
struct FwdCfg {
  static constexpr int kS = NS < 4 ? NS : 4;  // states per lane
  static constexpr int kLPC = NS / kS;        // lanes per channel
  static constexpr int kCPW = 32 / kLPC;      // channels per warp
  static constexpr int kWarps = kCh / kCPW;   // warps per CTA
  static constexpr int kThreads = kWarps * 32;
};

template <int NS, typename T>
struct FwdShared {
  // staging, written by TMA (two buffers)
  T rawD[2][kCh][kTile];
  T rawU[2][kCh][kTile];
  T rawZ[2][kCh][kTile];
  T rawB[2][NS][kTile];
  T rawC[2][NS][kTile];
  // fp32 work tiles
  float dlt[kCh][kRow];  // delta_eff
  float dlu[kCh][kRow];  // delta_eff * u   (ZOH: u)
  float ys[kCh][kRow];   // D u, then + sum_n C_t h_t
  float Bs[NS][kRow];
  float Cs[NS][kRow];
  uint64_t bar[2];
};

template <int NS, typename T, bool kZOH>
__global__ void __launch_bounds__(FwdCfg<NS>::kThreads)
    ss_fwd_kernel(const FwdParams p) {
  using Cfg = FwdCfg<NS>;
  constexpr int kS = Cfg::kS;
  constexpr int kLPC = Cfg::kLPC;
  constexpr int kThreads = Cfg::kThreads;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  FwdShared<NS, T>& sh = *reinterpret_cast<FwdShared<NS, T>*>(smem_raw);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int b = blockIdx.y;
  const int d0 = blockIdx.x * kCh;
  const int L = p.seqlen;
  const int n_ch = min(kCh, p.dim - d0);  // live channels of this CTA

  // this lane's channel slot and states (lane q owns states q, q+kLPC, ...)
  const int cl = warp * Cfg::kCPW + lane / kLPC;
  const int q = lane % kLPC;
  const bool lane_active = cl < n_ch;
  const int d = d0 + (lane_active ? cl : 0);
  const size_t row = static_cast<size_t>(b) * p.dim + d;

  int len = L;
  if (p.seq_lens) len = max(0, min(L, p.seq_lens[b]));

  float a2[kS], Av[kS], h[kS];
#pragma unroll
  for (int j = 0; j < kS; ++j) {
    const int n = q + kLPC * j;
    Av[j] = __ldg(p.A + d * NS + n);
    a2[j] = Av[j] * kLog2e;
    h[j] = (lane_active && p.h0) ? __ldg(p.h0 + row * NS + n) : 0.f;
  }

  const size_t bdl = static_cast<size_t>(b) * p.dim * L;
  const T* u_b = static_cast<const T*>(p.u) + bdl;
  const T* dl_b = static_cast<const T*>(p.delta) + bdl;
  const T* z_b = p.z ? static_cast<const T*>(p.z) + bdl : nullptr;
  T* out_b = static_cast<T*>(p.out) + bdl;
  T* pre_b = p.out_pre ? static_cast<T*>(p.out_pre) + bdl : nullptr;
  const T* B_b = static_cast<const T*>(p.B) + static_cast<size_t>(b) * NS * L;
  const T* C_b = static_cast<const T*>(p.C) + static_cast<size_t>(b) * NS * L;
  const bool use_tma = p.tma_ok != 0;

  // Issues the TMA copies of tile `k` into staging buffer k % 2.
  auto issue = [&](int k) {
    const int s = k & 1;
    const int t0 = k * kTile;
    uint64_t* bar = &sh.bar[s];
    if (t0 >= len) {
      mbar_arrive_expect_tx(bar, 0);
      return;
    }
    const uint32_t bytes = static_cast<uint32_t>(min(kTile, L - t0) * sizeof(T));
    const uint32_t rows = 2 * n_ch + (z_b ? n_ch : 0) + 2 * NS;
    mbar_arrive_expect_tx(bar, rows * bytes);
    for (int c = 0; c < n_ch; ++c) {
      const size_t off = static_cast<size_t>(d0 + c) * L + t0;
      tma_load_1d(&sh.rawD[s][c][0], dl_b + off, bytes, bar);
      tma_load_1d(&sh.rawU[s][c][0], u_b + off, bytes, bar);
      if (z_b) tma_load_1d(&sh.rawZ[s][c][0], z_b + off, bytes, bar);
    }
    for (int n = 0; n < NS; ++n) {
      const size_t off = static_cast<size_t>(n) * L + t0;
      tma_load_1d(&sh.rawB[s][n][0], B_b + off, bytes, bar);
      tma_load_1d(&sh.rawC[s][n][0], C_b + off, bytes, bar);
    }
  };

  const int n_tiles = (L + kTile - 1) / kTile;
  if (use_tma) {
    if (tid == 0) {
      mbar_init(&sh.bar[0], 1);
      mbar_init(&sh.bar[1], 1);
      fence_mbar_init();
      issue(0);
    }
    __syncthreads();
  }

  for (int k = 0; k < n_tiles; ++k) {
    const int s = k & 1;
    const int t0 = k * kTile;
    if (use_tma) {
      if (tid == 0 && k + 1 < n_tiles) {
        fence_proxy_async_smem();  // the previous reads of that buffer are done
        issue(k + 1);
      }
      const bool ok = mbar_wait_bounded(&sh.bar[s], (k >> 1) & 1);
      if (__syncthreads_or(!ok)) {
        // A copy never completed: report it, let the in-flight copies of the
        // other buffer finish (bounded), and leave.
        if (tid == 0) {
          atomicOr(&g_fwd_device_error, kErrTmaTimeout);
          if (k + 1 < n_tiles) mbar_wait_bounded(&sh.bar[s ^ 1], ((k + 1) >> 1) & 1);
        }
        return;
      }
    }

    if (t0 < len) {
      // ---- 1. transform the tile into fp32 work tiles
      for (int i = tid; i < kCh * kTile; i += kThreads) {
        const int c = i / kTile, tt = i % kTile;
        const int t = t0 + tt;
        float dv = 0.f, du = 0.f, yd = 0.f;
        if (c < n_ch && t < len) {
          float x, uv;
          if (use_tma) {
            x = to_f32(sh.rawD[s][c][tt]);
            uv = to_f32(sh.rawU[s][c][tt]);
          } else {
            const size_t off = static_cast<size_t>(d0 + c) * L + t;
            x = Elem<T>::ld(dl_b + off);
            uv = Elem<T>::ld(u_b + off);
          }
          if (p.delta_bias) x += __ldg(p.delta_bias + d0 + c);
          dv = p.delta_softplus ? softplus_f(x) : x;
          du = kZOH ? uv : dv * uv;
          if (p.D) yd = __ldg(p.D + d0 + c) * uv;
        }
        sh.dlt[c][tt] = dv;
        sh.dlu[c][tt] = du;
        sh.ys[c][tt] = yd;
      }
      for (int i = tid; i < NS * kTile; i += kThreads) {
        const int n = i / kTile, tt = i % kTile;
        const int t = t0 + tt;
        float bv = 0.f, cv = 0.f;
        if (t < len) {
          if (use_tma) {
            bv = to_f32(sh.rawB[s][n][tt]);
            cv = to_f32(sh.rawC[s][n][tt]);
          } else {
            bv = Elem<T>::ld(B_b + static_cast<size_t>(n) * L + t);
            cv = Elem<T>::ld(C_b + static_cast<size_t>(n) * L + t);
          }
        }
        sh.Bs[n][tt] = bv;
        sh.Cs[n][tt] = cv;
      }
      __syncthreads();

      // ---- 2. sequential scan over the tile, 4 steps per iteration; the
      // kLPC lanes of a channel read adjacent B/C rows (distinct banks) and
      // pairs of steps are packed into fp32x2 operations.
      const int steps = min(kTile, len - t0);
#pragma unroll 2
      for (int tt = 0; tt < steps; tt += 4) {
        const float4 dl4 = *reinterpret_cast<const float4*>(&sh.dlt[cl][tt]);
        const float4 du4 = *reinterpret_cast<const float4*>(&sh.dlu[cl][tt]);
        const float2 dlp[2] = {make_float2(dl4.x, dl4.y), make_float2(dl4.z, dl4.w)};
        const float2 dup_[2] = {make_float2(du4.x, du4.y), make_float2(du4.z, du4.w)};
        float2 yp2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int j = 0; j < kS; ++j) {
          const int n = q + kLPC * j;
          const float4 B4 = *reinterpret_cast<const float4*>(&sh.Bs[n][tt]);
          const float4 C4 = *reinterpret_cast<const float4*>(&sh.Cs[n][tt]);
          const float2 Bp[2] = {make_float2(B4.x, B4.y), make_float2(B4.z, B4.w)};
          const float2 Cp[2] = {make_float2(C4.x, C4.y), make_float2(C4.z, C4.w)};
          const float2 a2p = dup2(a2[j]);
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float2 arg = mul2(dlp[e], a2p);
            const float2 ab = make_float2(ex2(arg.x), ex2(arg.y));
            float2 bu;
            if constexpr (kZOH) {
              // b_bar = expm1(delta*A) / A * B   (mamba/selective_scan_cuda.py:77)
              const float inv = 1.f / Av[j];
              bu.x = Bp[e].x * (expm1f(dlp[e].x * Av[j]) * inv) * dup_[e].x;
              bu.y = Bp[e].y * (expm1f(dlp[e].y * Av[j]) * inv) * dup_[e].y;
            } else {
              bu = mul2(Bp[e], dup_[e]);
            }
            float2 hh;
            hh.x = h[j] = fmaf(ab.x, h[j], bu.x);
            hh.y = h[j] = fmaf(ab.y, h[j], bu.y);
            yp2[e] = fma2(Cp[e], hh, yp2[e]);
          }
        }
        const float yp[4] = {yp2[0].x, yp2[0].y, yp2[1].x, yp2[1].y};
        // sum the kLPC lanes of a channel (reduce-scatter: lane q keeps the
        // steps it will store)
        if constexpr (kLPC == 4) {
          const bool hi2 = (q & 2) != 0;
          const float s0 = hi2 ? yp[0] : yp[2], s1 = hi2 ? yp[1] : yp[3];
          float k0 = hi2 ? yp[2] : yp[0], k1 = hi2 ? yp[3] : yp[1];
          k0 += __shfl_xor_sync(0xffffffffu, s0, 2);
          k1 += __shfl_xor_sync(0xffffffffu, s1, 2);
          const bool hi1 = (q & 1) != 0;
          const float sx = hi1 ? k0 : k1;
          float kk = hi1 ? k1 : k0;
          kk += __shfl_xor_sync(0xffffffffu, sx, 1);
          sh.ys[cl][tt + q] += kk;  // step tt + q
        } else if constexpr (kLPC == 2) {
          const bool hi = (q & 1) != 0;
          const float s0 = hi ? yp[0] : yp[2], s1 = hi ? yp[1] : yp[3];
          float k0 = hi ? yp[2] : yp[0], k1 = hi ? yp[3] : yp[1];
          k0 += __shfl_xor_sync(0xffffffffu, s0, 1);
          k1 += __shfl_xor_sync(0xffffffffu, s1, 1);
          sh.ys[cl][tt + 2 * q] += k0;
          sh.ys[cl][tt + 2 * q + 1] += k1;
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) sh.ys[cl][tt + e] += yp[e];
        }
      }
    }

    // ---- carry checkpoint at the end of every chunk (and of the sequence)
    const int t_end = t0 + kTile;
    if (lane_active && (t_end % kChunk == 0 || t_end >= L)) {
      const int c = (t_end - 1) / kChunk;
#pragma unroll
      for (int j = 0; j < kS; ++j)
        p.chunk_states[(row * p.n_chunks + c) * NS + q + kLPC * j] = h[j];
    }
    __syncthreads();

    // ---- 3. emit out = (y + D u) * silu(z), and y + D u
    for (int i = tid; i < kCh * kTile; i += kThreads) {
      const int c = i / kTile, tt = i % kTile;
      const int t = t0 + tt;
      if (c >= n_ch || t >= L) continue;
      const size_t off = static_cast<size_t>(d0 + c) * L + t;
      float o = 0.f, pre = 0.f;
      if (t < len) {
        pre = sh.ys[c][tt];
        if (z_b) {
          const float zv = use_tma ? to_f32(sh.rawZ[s][c][tt]) : Elem<T>::ld(z_b + off);
          o = pre * silu_f(zv);
        } else {
          o = pre;
        }
      }
      Elem<T>::st(out_b + off, o);
      if (pre_b) Elem<T>::st(pre_b + off, pre);
    }
    __syncthreads();
  }

  if (p.last_state && lane_active) {
#pragma unroll
    for (int j = 0; j < kS; ++j) p.last_state[row * NS + q + kLPC * j] = h[j];
  }
}

template <int NS, typename T, bool kZOH>
static cudaError_t launch_fwd_t(const FwdParams& p, cudaStream_t stream) {
  using Cfg = FwdCfg<NS>;
  const size_t smem = sizeof(FwdShared<NS, T>);
  auto kern = ss_fwd_kernel<NS, T, kZOH>;
  cudaError_t e = cudaFuncSetAttribute(
      kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  dim3 grid((p.dim + kCh - 1) / kCh, p.batch);
  kern<<<grid, Cfg::kThreads, smem, stream>>>(p);
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

static bool aligned16(const void* ptr) {
  return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0;
}

cudaError_t launch_fwd(const FwdParams& p_in, int dstate, int io_dtype, int zoh,
                       cudaStream_t stream) {
  FwdParams p = p_in;
  const size_t esize = io_dtype == MSS_BF16 ? 2 : 4;
  // TMA rows need 16-byte aligned starts and sizes: whole rows of L elements
  // and tiles of kTile elements must both be multiples of 16 bytes.
  p.tma_ok = (p.seqlen * esize) % 16 == 0 && aligned16(p.u) && aligned16(p.delta) &&
             aligned16(p.B) && aligned16(p.C) && (!p.z || aligned16(p.z));
  if (io_dtype == MSS_BF16) {
    return zoh ? launch_fwd_n<__nv_bfloat16, true>(p, dstate, stream)
               : launch_fwd_n<__nv_bfloat16, false>(p, dstate, stream);
  }
  return zoh ? launch_fwd_n<float, true>(p, dstate, stream)
             : launch_fwd_n<float, false>(p, dstate, stream);
}

unsigned int take_fwd_device_error() {
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_fwd_device_error, sizeof(v)) != cudaSuccess) return ~0u;
  cudaMemcpyToSymbol(g_fwd_device_error, &zero, sizeof(zero));
  return v;
}

}  // namespace mss

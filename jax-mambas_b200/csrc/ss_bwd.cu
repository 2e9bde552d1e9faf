// Backward selective scan for sm_100a.
//
// Replaces selective_scan_bwd_kernel (native/upstream_mamba/
// selective_scan_bwd_kernel.cuh:65-497) and SelectiveScanBackwardImpl
// (native/selective_scan_bwd.cu:24-162), and adds the gradients of the fused
// softplus(delta + bias), D skip and silu(z) gate, and the ZOH discretization
// the reference leaves to JAX autodiff (mamba/selective_scan_cuda.py:250-256).
//
// Per (batch, channel) row a warp walks the chunks in reverse. For each chunk
// and state it
//   1. recomputes h_{t-1} over the chunk from the saved carry (forward scan),
//   2. runs the adjoint recurrence g_t = dy_t C_t + a_{t+1} g_{t+1} as a
//      reverse warp scan seeded with the carry from the later chunk,
//   3. accumulates ddelta, du (per row), dA (per lane, shared memory) and the
//      cross-channel sums dB, dC in a shared-memory tile.
// dB/dC sum over the channels of a batch. The warps of a CTA (channels of one
// batch) fold into one shared tile without atomics: at step s warp w works on
// state (s + w*NS/G) mod NS, so no two warps touch one state row between the
// barriers placed every NS/G steps. At the end of a chunk the tile is added
// to the fp32 accumulators in global memory with 16-byte atomics.
#include "ss_common.cuh"
#include "ss_launch.h"

namespace mss {

constexpr int kBwdWarps = 4;

// Column of logical step tc (multiple of 4) inside a shared tile row. Lanes
// write 32-byte runs; flipping the 16-byte half for lanes 4..7 (mod 8) keeps
// each quarter-warp of 128-bit accesses on distinct banks.
__device__ __forceinline__ int tile_col(int tc) {
  const int i = tc >> 3;
  const int g = (tc >> 2) & 1;
  return (i << 3) + ((g ^ ((i >> 2) & 1)) << 2);
}

template <int NS>
struct BwdShared {
  static constexpr int G = NS < kBwdWarps ? NS : kBwdWarps;  // warps per copy
  static constexpr int R = kBwdWarps / G;                    // tile copies
  float accB[R][NS][kChunk];
  float accC[R][NS][kChunk];
  float gcarry[kBwdWarps][NS];
  float dA[kBwdWarps][NS][32];
};

template <int NS, typename T, bool kZOH>
__global__ void __launch_bounds__(kBwdWarps * 32)
    ss_bwd_kernel(const BwdParams p) {
  using Sh = BwdShared<NS>;
  constexpr int G = Sh::G;
  constexpr int R = Sh::R;
  constexpr int kPhase = NS / G;  // steps between barriers
  __shared__ __align__(16) Sh sh;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int d = blockIdx.x * kBwdWarps + warp;
  const int b = blockIdx.y;
  const bool active = d < p.dim;
  const int dc = active ? d : 0;  // clamp for parameter loads
  const int copy = warp / G;
  const int rot = (warp % G) * kPhase;

  const int L = p.seqlen;
  const size_t row = static_cast<size_t>(b) * p.dim + dc;
  const T* u_row = static_cast<const T*>(p.u) + row * L;
  const T* dl_row = static_cast<const T*>(p.delta) + row * L;
  const T* z_row = p.z ? static_cast<const T*>(p.z) + row * L : nullptr;
  const T* dout_row = static_cast<const T*>(p.dout) + row * L;
  T* du_row = static_cast<T*>(p.du) + row * L;
  T* ddl_row = static_cast<T*>(p.ddelta) + row * L;
  T* dz_row = p.dz ? static_cast<T*>(p.dz) + row * L : nullptr;
  const T* B_b = static_cast<const T*>(p.B) + static_cast<size_t>(b) * NS * L;
  const T* C_b = static_cast<const T*>(p.C) + static_cast<size_t>(b) * NS * L;

  int len = L;
  if (p.seq_lens) len = max(0, min(L, p.seq_lens[b]));
  const int lim = active ? len : 0;  // inactive warps see zeros
  const float Dv = p.D ? __ldg(p.D + dc) : 0.f;
  const float bias = p.delta_bias ? __ldg(p.delta_bias + dc) : 0.f;

  // Zero the tiles, seed the adjoint carries, clear the dA partials.
  for (int i = threadIdx.x; i < R * NS * kChunk; i += blockDim.x) {
    (&sh.accB[0][0][0])[i] = 0.f;
    (&sh.accC[0][0][0])[i] = 0.f;
  }
  if (lane < NS) {
    sh.gcarry[warp][lane] =
        (active && p.dlast) ? __ldg(p.dlast + row * NS + lane) : 0.f;
  }
#pragma unroll
  for (int n = 0; n < NS; ++n) sh.dA[warp][n][lane] = 0.f;
  __syncthreads();

  float dD_acc = 0.f, dbias_acc = 0.f;

  for (int c = p.n_chunks - 1; c >= 0; --c) {
    const int t0 = c * kChunk;
    const int tl = t0 + lane * kItems;

    if (t0 >= len) {
      // Padding-only chunk (CTA-uniform: len depends on the batch only).
      if (active) {
        float zero[kItems];
#pragma unroll
        for (int k = 0; k < kItems; ++k) zero[k] = 0.f;
        store_run(du_row, tl, L, zero);
        store_run(ddl_row, tl, L, zero);
        if (dz_row) store_run(dz_row, tl, L, zero);
      }
      continue;
    }

    float uv[kItems], dl[kItems], dv[kItems], dy[kItems], dzf[kItems];
    load_run(u_row, tl, lim, uv);
    load_run(dl_row, tl, lim, dl);
    load_run(dout_row, tl, lim, dy);
    if (z_row) {
      float zv[kItems];
      load_run(z_row, tl, lim, zv);
#pragma unroll
      for (int k = 0; k < kItems; ++k) {
        const float sg = sigmoid(zv[k]);
        const float silu = zv[k] * sg;
        dzf[k] = dy[k] * sg * (1.f + zv[k] * (1.f - sg));  // dout * silu'(z)
        dy[k] *= silu;
      }
    }
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      const bool valid = tl + k < lim;
      dv[k] = dl[k] + bias;  // pre-activation, kept for the softplus gradient
      float v = p.delta_softplus ? softplus(dv[k]) : dv[k];
      dl[k] = valid ? v : 0.f;
    }

    float y[kItems], ddl[kItems], dua[kItems], duv[kItems];
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      y[k] = 0.f;
      ddl[k] = 0.f;
      dua[k] = 0.f;
      duv[k] = dl[k] * uv[k];
    }

#pragma unroll 1
    for (int s = 0; s < NS; ++s) {
      const int n = (s + rot) % NS;
      const float An = __ldg(p.A + dc * NS + n);
      const float a2 = An * kLog2e;
      float hs;
      if (c == 0)
        hs = (p.h0 && active) ? __ldg(p.h0 + row * NS + n) : 0.f;
      else
        hs = active ? p.chunk_states[(row * p.n_chunks + c - 1) * NS + n] : 0.f;

      float Bv[kItems], Cv[kItems];
      load_run(B_b + static_cast<size_t>(n) * L, tl, lim, Bv);
      load_run(C_b + static_cast<size_t>(n) * L, tl, lim, Cv);

      // ---- forward recompute of h_{t-1}
      float ab[kItems], bu[kItems], bb[kItems];
      float P = 1.f, H = 0.f;
#pragma unroll
      for (int k = 0; k < kItems; ++k) {
        ab[k] = ex2(dl[k] * a2);
        if constexpr (kZOH) {
          bb[k] = expm1f(dl[k] * An) * (1.f / An);
          bu[k] = Bv[k] * bb[k] * uv[k];
        } else {
          bu[k] = Bv[k] * duv[k];
        }
        H = fmaf(ab[k], H, bu[k]);
        P *= ab[k];
      }
      warp_scan_fwd(P, H, lane);
      {
        float Pe = __shfl_up_sync(0xffffffffu, P, 1);
        float He = __shfl_up_sync(0xffffffffu, H, 1);
        if (lane == 0) {
          Pe = 1.f;
          He = 0.f;
        }
        H = fmaf(Pe, hs, He);  // h entering this lane's run
      }
      float hp[kItems], dCv[kItems];
      {
        float h = H;
#pragma unroll
        for (int k = 0; k < kItems; ++k) {
          hp[k] = h;
          h = fmaf(ab[k], h, bu[k]);
          y[k] = fmaf(Cv[k], h, y[k]);
          dCv[k] = dy[k] * h;
        }
      }

      // ---- adjoint: g_t = dy_t C_t + a_{t+1} g_{t+1}
      float an[kItems];
#pragma unroll
      for (int k = 0; k < kItems - 1; ++k) an[k] = ab[k + 1];
      an[kItems - 1] = __shfl_down_sync(0xffffffffu, ab[0], 1);
      if (lane == 31) an[kItems - 1] = 1.f;  // the carry already holds a g
      float Pr = 1.f, Gr = 0.f;
#pragma unroll
      for (int k = kItems - 1; k >= 0; --k) {
        Gr = fmaf(an[k], Gr, dy[k] * Cv[k]);
        Pr *= an[k];
      }
      warp_scan_rev(Pr, Gr, lane);
      float Pe = __shfl_down_sync(0xffffffffu, Pr, 1);
      float Ge = __shfl_down_sync(0xffffffffu, Gr, 1);
      if (lane == 31) {
        Pe = 1.f;
        Ge = 0.f;
      }
      float g = fmaf(Pe, sh.gcarry[warp][n], Ge);
      float dAl = 0.f;
      float dBv[kItems];
#pragma unroll
      for (int k = kItems - 1; k >= 0; --k) {
        g = fmaf(an[k], g, dy[k] * Cv[k]);
        const float w = g * hp[k] * ab[k];  // g_t a_t h_{t-1}
        if constexpr (kZOH) {
          ddl[k] += g * ab[k] * Bv[k] * uv[k] + w * An;
          dua[k] = fmaf(g * bb[k], Bv[k], dua[k]);
          dBv[k] = g * bb[k] * uv[k];
          dAl += w * dl[k] +
                 g * Bv[k] * uv[k] * (dl[k] * ab[k] - bb[k]) * (1.f / An);
        } else {
          ddl[k] += fmaf(g * Bv[k], uv[k], w * An);
          dua[k] = fmaf(g, Bv[k], dua[k]);
          dBv[k] = g * duv[k];
          dAl = fmaf(w, dl[k], dAl);
        }
      }
      const float gnext = __shfl_sync(0xffffffffu, ab[0] * g, 0);
      if (lane == 0) sh.gcarry[warp][n] = gnext;
      sh.dA[warp][n][lane] += dAl;

      // ---- fold dB/dC into this warp's tile row (owned until the barrier)
      {
        float4* rb = reinterpret_cast<float4*>(&sh.accB[copy][n][0]);
        float4* rc = reinterpret_cast<float4*>(&sh.accC[copy][n][0]);
#pragma unroll
        for (int q = 0; q < kItems / 4; ++q) {
          const int col = tile_col(lane * kItems + 4 * q) >> 2;
          float4 vb = rb[col], vc = rc[col];
          vb.x += dBv[4 * q + 0]; vb.y += dBv[4 * q + 1];
          vb.z += dBv[4 * q + 2]; vb.w += dBv[4 * q + 3];
          vc.x += dCv[4 * q + 0]; vc.y += dCv[4 * q + 1];
          vc.z += dCv[4 * q + 2]; vc.w += dCv[4 * q + 3];
          rb[col] = vb;
          rc[col] = vc;
        }
      }
      if ((s + 1) % kPhase == 0) __syncthreads();
    }

    // ---- flush the dB/dC tiles of this chunk into global fp32 accumulators
    {
      const size_t base = static_cast<size_t>(b) * NS * L;
      for (int q = threadIdx.x; q < NS * (kChunk / 4); q += blockDim.x) {
        const int n = q / (kChunk / 4);
        const int tc = (q % (kChunk / 4)) * 4;
        const int col = tile_col(tc);
        float4 vb = make_float4(0.f, 0.f, 0.f, 0.f), vc = vb;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const float4 xb = *reinterpret_cast<const float4*>(&sh.accB[r][n][col]);
          const float4 xc = *reinterpret_cast<const float4*>(&sh.accC[r][n][col]);
          vb.x += xb.x; vb.y += xb.y; vb.z += xb.z; vb.w += xb.w;
          vc.x += xc.x; vc.y += xc.y; vc.z += xc.z; vc.w += xc.w;
          *reinterpret_cast<float4*>(&sh.accB[r][n][col]) =
              make_float4(0.f, 0.f, 0.f, 0.f);
          *reinterpret_cast<float4*>(&sh.accC[r][n][col]) =
              make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const int t = t0 + tc;
        if (t >= len) continue;
        float* gb = p.dB_acc + base + static_cast<size_t>(n) * L + t;
        float* gc = p.dC_acc + base + static_cast<size_t>(n) * L + t;
        if (t + 4 <= len && ((reinterpret_cast<uintptr_t>(gb) & 15) == 0) &&
            ((reinterpret_cast<uintptr_t>(gc) & 15) == 0)) {
          atomicAdd(reinterpret_cast<float4*>(gb), vb);
          atomicAdd(reinterpret_cast<float4*>(gc), vc);
        } else {
          const float eb[4] = {vb.x, vb.y, vb.z, vb.w};
          const float ec[4] = {vc.x, vc.y, vc.z, vc.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (t + e < len) {
              atomicAdd(gb + e, eb[e]);
              atomicAdd(gc + e, ec[e]);
            }
          }
        }
      }
      __syncthreads();
    }

    // ---- per-element epilogue
    if (active) {
      float zv[kItems];
      if (z_row) load_run(z_row, tl, lim, zv);
      float o_du[kItems], o_dd[kItems], o_dz[kItems];
#pragma unroll
      for (int k = 0; k < kItems; ++k) {
        const bool valid = tl + k < lim;
        float gd = ddl[k];
        if (p.delta_softplus) gd *= sigmoid(dv[k]);
        gd = valid ? gd : 0.f;
        const float gu = kZOH ? dua[k] : dl[k] * dua[k];
        o_dd[k] = gd;
        o_du[k] = valid ? fmaf(Dv, dy[k], gu) : 0.f;
        o_dz[k] = (z_row && valid) ? dzf[k] * fmaf(Dv, uv[k], y[k]) : 0.f;
        dD_acc = fmaf(dy[k], uv[k], dD_acc);
        dbias_acc += gd;
      }
      store_run(du_row, tl, L, o_du);
      store_run(ddl_row, tl, L, o_dd);
      if (dz_row) store_run(dz_row, tl, L, o_dz);
    }
  }

  // ---- per-row results
  dD_acc = warp_sum(dD_acc);
  dbias_acc = warp_sum(dbias_acc);
  float dAv[NS];
#pragma unroll
  for (int n = 0; n < NS; ++n) dAv[n] = warp_sum(sh.dA[warp][n][lane]);
  if (active && lane == 0) {
#pragma unroll
    for (int n = 0; n < NS; ++n) {
      p.dA_part[row * NS + n] = dAv[n];
      if (p.dh0) p.dh0[row * NS + n] = sh.gcarry[warp][n];
    }
    p.dD_part[row] = dD_acc;
    p.dbias_part[row] = dbias_acc;
  }
}

// Sums the per-batch partials of dA (dim*dstate), dD and ddelta_bias (dim)
// in a fixed order, so these three are bitwise reproducible.
__global__ void reduce_params_kernel(const float* __restrict__ dA_part,
                                     const float* __restrict__ dD_part,
                                     const float* __restrict__ dbias_part,
                                     float* dA, float* dD, float* dbias,
                                     int batch, int dim, int dstate) {
  const int nA = dim * dstate;
  const int total = nA + 2 * dim;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += gridDim.x * blockDim.x) {
    if (i < nA) {
      float s = 0.f;
      for (int b = 0; b < batch; ++b) s += dA_part[static_cast<size_t>(b) * nA + i];
      dA[i] = s;
    } else if (i < nA + dim) {
      const int j = i - nA;
      if (dD) {
        float s = 0.f;
        for (int b = 0; b < batch; ++b) s += dD_part[static_cast<size_t>(b) * dim + j];
        dD[j] = s;
      }
    } else {
      const int j = i - nA - dim;
      if (dbias) {
        float s = 0.f;
        for (int b = 0; b < batch; ++b) s += dbias_part[static_cast<size_t>(b) * dim + j];
        dbias[j] = s;
      }
    }
  }
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ src,
                                   __nv_bfloat16* __restrict__ dst, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
       i < n; i += static_cast<size_t>(gridDim.x) * blockDim.x)
    dst[i] = __float2bfloat16_rn(src[i]);
}

template <int NS, typename T, bool kZOH>
static cudaError_t launch_bwd_t(const BwdParams& p, cudaStream_t stream) {
  dim3 grid((p.dim + kBwdWarps - 1) / kBwdWarps, p.batch);
  ss_bwd_kernel<NS, T, kZOH><<<grid, kBwdWarps * 32, 0, stream>>>(p);
  return cudaPeekAtLastError();
}

template <typename T, bool kZOH>
static cudaError_t launch_bwd_n(const BwdParams& p, int dstate,
                                cudaStream_t stream) {
  switch (dstate) {
    case 1: return launch_bwd_t<1, T, kZOH>(p, stream);
    case 2: return launch_bwd_t<2, T, kZOH>(p, stream);
    case 4: return launch_bwd_t<4, T, kZOH>(p, stream);
    case 8: return launch_bwd_t<8, T, kZOH>(p, stream);
    case 16: return launch_bwd_t<16, T, kZOH>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_bwd(const BwdParams& p, int dstate, int io_dtype, int zoh,
                       void* dB_out, void* dC_out, float* dA, float* dD,
                       float* ddelta_bias, cudaStream_t stream) {
  const size_t n_bnl = static_cast<size_t>(p.batch) * dstate * p.seqlen;
  cudaError_t e = cudaMemsetAsync(p.dB_acc, 0, n_bnl * sizeof(float), stream);
  if (e != cudaSuccess) return e;
  e = cudaMemsetAsync(p.dC_acc, 0, n_bnl * sizeof(float), stream);
  if (e != cudaSuccess) return e;

  if (io_dtype == MSS_BF16) {
    e = zoh ? launch_bwd_n<__nv_bfloat16, true>(p, dstate, stream)
            : launch_bwd_n<__nv_bfloat16, false>(p, dstate, stream);
  } else {
    e = zoh ? launch_bwd_n<float, true>(p, dstate, stream)
            : launch_bwd_n<float, false>(p, dstate, stream);
  }
  if (e != cudaSuccess) return e;

  {
    const int total = p.dim * dstate + 2 * p.dim;
    const int threads = 256;
    const int blocks = (total + threads - 1) / threads;
    reduce_params_kernel<<<blocks, threads, 0, stream>>>(
        p.dA_part, p.dD_part, p.dbias_part, dA, dD, ddelta_bias, p.batch,
        p.dim, dstate);
    e = cudaPeekAtLastError();
    if (e != cudaSuccess) return e;
  }
  if (io_dtype == MSS_BF16) {
    const int threads = 256;
    const int blocks = static_cast<int>(
        std::min<size_t>((n_bnl + threads - 1) / threads, 148 * 16));
    f32_to_bf16_kernel<<<blocks, threads, 0, stream>>>(
        p.dB_acc, static_cast<__nv_bfloat16*>(dB_out), n_bnl);
    f32_to_bf16_kernel<<<blocks, threads, 0, stream>>>(
        p.dC_acc, static_cast<__nv_bfloat16*>(dC_out), n_bnl);
    e = cudaPeekAtLastError();
  }
  return e;
}

}  // namespace mss

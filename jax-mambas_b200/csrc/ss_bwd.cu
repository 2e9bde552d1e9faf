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
//   1. recomputes h_t over the chunk from the saved carry (forward scan),
//   2. runs the adjoint recurrence g_t = dy_t C_t + a_{t+1} g_{t+1} as a
//      reverse warp scan seeded with the carry from the later chunk,
//   3. accumulates, per step, sum_n g B (-> du, and the u-part of ddelta),
//      sum_n g a h_{t-1} A (-> ddelta), per lane dA, and the cross-channel
//      sums dB = g delta u and dC = dy h in a shared-memory tile.
// dz uses the pre-gate output y + D u saved by the forward.
// dB/dC sum over the channels of a batch. The warps of a CTA (channels of one
// batch) fold into one shared tile without atomics: at step s warp w works on
// state (s + w*NS/G) mod NS, so no two warps touch one state row between the
// barriers placed every NS/G steps. At the end of a chunk the tile is added
// to the fp32 accumulators in global memory with 16-byte atomics.
#include <algorithm>

#include "ss_common.cuh"
#include "ss_launch.h"

namespace mss {

constexpr int kBwdWarps = 4;
constexpr int kHalf = kItems / 2;

// Float4 slot of logical float4 group q (q = t_in_chunk / 4) in a shared tile
// row. Lane i writes the four groups 4i..4i+3; XOR-ing the group index with
// (i >> 1) & 3 spreads each quarter-warp of 128-bit accesses over all banks.
__device__ __forceinline__ int tile_slot(int q) {
  const int i = q >> 2;
  return (i << 2) | ((q & 3) ^ ((i >> 1) & 3));
}

template <int NS>
struct BwdShared {
  static constexpr int G = NS < kBwdWarps ? NS : kBwdWarps;  // warps per copy
  static constexpr int R = kBwdWarps / G;                    // tile copies
  float4 accB[R][NS][kChunk / 4];
  float4 accC[R][NS][kChunk / 4];
  float gcarry[kBwdWarps][NS];
  float dA[kBwdWarps][NS][32];
};

template <int NS, typename T, bool kZOH>
__global__ void __launch_bounds__(kBwdWarps * 32, 3)
    ss_bwd_kernel(const BwdParams p) {
  using Sh = BwdShared<NS>;
  constexpr int G = Sh::G;
  constexpr int R = Sh::R;
  constexpr int kPhase = NS / G;  // steps between barriers
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Sh& sh = *reinterpret_cast<Sh*>(smem_raw);

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
  for (int i = threadIdx.x; i < R * NS * (kChunk / 4); i += blockDim.x) {
    (&sh.accB[0][0][0])[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    (&sh.accC[0][0][0])[i] = make_float4(0.f, 0.f, 0.f, 0.f);
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
        float2 zero[kHalf];
#pragma unroll
        for (int i = 0; i < kHalf; ++i) zero[i] = make_float2(0.f, 0.f);
        store_run2(du_row, tl, L, zero);
        store_run2(ddl_row, tl, L, zero);
        if (dz_row) store_run2(dz_row, tl, L, zero);
      }
      continue;
    }

    // ---- per-step inputs of this lane's run
    float2 dl[kHalf], duv[kHalf], dy[kHalf];
    float ssum, ssum1;  // sum of delta over the run, and without its first step
    {
      float2 uv[kHalf];
      load_run2(u_row, tl, lim, uv);
      load_run2(dl_row, tl, lim, dl);
      load_run2(dout_row, tl, lim, dy);
      if (z_row) {
        float2 zv[kHalf];
        load_run2(z_row, tl, lim, zv);
#pragma unroll
        for (int i = 0; i < kHalf; ++i) {
          dy[i].x *= silu_f(zv[i].x);
          dy[i].y *= silu_f(zv[i].y);
        }
      }
      ssum = 0.f;
#pragma unroll
      for (int i = 0; i < kHalf; ++i) {
        float v0 = dl[i].x + bias, v1 = dl[i].y + bias;
        if (p.delta_softplus) {
          v0 = softplus_f(v0);
          v1 = softplus_f(v1);
        }
        dl[i].x = (tl + 2 * i < lim) ? v0 : 0.f;
        dl[i].y = (tl + 2 * i + 1 < lim) ? v1 : 0.f;
        ssum += dl[i].x + dl[i].y;
        duv[i] = kZOH ? uv[i] : mul2(dl[i], uv[i]);
      }
      ssum1 = ssum - dl[0].x;
    }

    float2 gA[kHalf], gB[kHalf];
#pragma unroll
    for (int i = 0; i < kHalf; ++i) {
      gA[i] = make_float2(0.f, 0.f);  // sum_n g a h_{t-1} A_n  (ZOH: + g a B u)
      gB[i] = make_float2(0.f, 0.f);  // sum_n g B_n            (ZOH: g b_bar)
    }

#pragma unroll 1
    for (int s = 0; s < NS; ++s) {
      const int n = (s + rot) % NS;
      const float An = __ldg(p.A + dc * NS + n);
      const float2 a2 = dup2(An * kLog2e);
      const float2 A2 = dup2(An);
      float hs;
      if (c == 0)
        hs = (p.h0 && active) ? __ldg(p.h0 + row * NS + n) : 0.f;
      else
        hs = active ? p.chunk_states[(row * p.n_chunks + c - 1) * NS + n] : 0.f;
      const T* Bn = B_b + static_cast<size_t>(n) * L;
      const T* Cn = C_b + static_cast<size_t>(n) * L;
      float4* tileB = &sh.accB[copy][n][0];
      float4* tileC = &sh.accC[copy][n][0];

      // ---- forward recompute: a_t, and h_t for every step of the run
      float2 ab[kHalf], hv[kHalf];
      {
        float2 Bv[kHalf];
        load_run2(Bn, tl, lim, Bv);
        float H = 0.f;
#pragma unroll
        for (int i = 0; i < kHalf; ++i) {
          const float2 arg = mul2(dl[i], a2);
          ab[i] = make_float2(ex2(arg.x), ex2(arg.y));
          float2 bu;
          if constexpr (kZOH) {
            const float inv = 1.f / An;
            bu.x = Bv[i].x * (expm1f(dl[i].x * An) * inv) * duv[i].x;
            bu.y = Bv[i].y * (expm1f(dl[i].y * An) * inv) * duv[i].y;
          } else {
            bu = mul2(Bv[i], duv[i]);
          }
          hv[i] = bu;  // b_t for now; h_t after the re-walk
          H = fmaf(ab[i].x, H, bu.x);
          H = fmaf(ab[i].y, H, bu.y);
        }
        float P = ex2(a2.x * ssum);
        warp_scan_fwd(P, H, lane);
        float Pe = __shfl_up_sync(0xffffffffu, P, 1);
        float He = __shfl_up_sync(0xffffffffu, H, 1);
        if (lane == 0) {
          Pe = 1.f;
          He = 0.f;
        }
        float h = fmaf(Pe, hs, He);  // h entering this lane's run
#pragma unroll
        for (int i = 0; i < kHalf; ++i) {
          hv[i].x = h = fmaf(ab[i].x, h, hv[i].x);
          hv[i].y = h = fmaf(ab[i].y, h, hv[i].y);
        }
      }

      // ---- dC = dy h (folded into the tile now) and e_t = dy_t C_t
      float2 ev[kHalf];
      {
        float2 Cv[kHalf];
        load_run2(Cn, tl, lim, Cv);
#pragma unroll
        for (int j = 0; j < kItems / 4; ++j) {
          ev[2 * j] = mul2(dy[2 * j], Cv[2 * j]);
          ev[2 * j + 1] = mul2(dy[2 * j + 1], Cv[2 * j + 1]);
          const float2 c0 = mul2(dy[2 * j], hv[2 * j]);
          const float2 c1 = mul2(dy[2 * j + 1], hv[2 * j + 1]);
          float4& slot = tileC[tile_slot(lane * (kItems / 4) + j)];
          const float4 v = slot;
          const float2 lo = add2(make_float2(v.x, v.y), c0);
          const float2 hi = add2(make_float2(v.z, v.w), c1);
          slot = make_float4(lo.x, lo.y, hi.x, hi.y);
        }
      }

      // ---- adjoint scan: g_t = e_t + a_{t+1} g_{t+1}
      float an_last = __shfl_down_sync(0xffffffffu, ab[0].x, 1);
      if (lane == 31) an_last = 1.f;  // the carry already holds a_{t+1} g_{t+1}
      float g;
      {
        float Gr = ev[kHalf - 1].y;
        Gr = fmaf(ab[kHalf - 1].y, Gr, ev[kHalf - 1].x);
#pragma unroll
        for (int i = kHalf - 2; i >= 0; --i) {
          Gr = fmaf(ab[i + 1].x, Gr, ev[i].y);
          Gr = fmaf(ab[i].y, Gr, ev[i].x);
        }
        // lane map g_next -> Pr g_next + Gr with Pr = a_1 ... a_15 a_next
        float Pr = ex2(a2.x * ssum1) * an_last;
        warp_scan_rev(Pr, Gr, lane);
        float Pe = __shfl_down_sync(0xffffffffu, Pr, 1);
        float Ge = __shfl_down_sync(0xffffffffu, Gr, 1);
        if (lane == 31) {
          Pe = 1.f;
          Ge = 0.f;
        }
        g = fmaf(Pe, sh.gcarry[warp][n], Ge);  // g of the next lane's first step
      }

      // ---- re-walk g backwards and form the gradient terms
      float2 dAl = make_float2(0.f, 0.f);
      {
        float2 Bv[kHalf];
        load_run2(Bn, tl, lim, Bv);
        float2 db_hi = make_float2(0.f, 0.f);
#pragma unroll
        for (int i = kHalf - 1; i >= 0; --i) {
          float2 gv;
          gv.y = g = fmaf(i == kHalf - 1 ? an_last : ab[i + 1].x, g, ev[i].y);
          gv.x = g = fmaf(ab[i].y, g, ev[i].x);
          float2 bu, bb;
          if constexpr (kZOH) {
            const float inv = 1.f / An;
            bb.x = expm1f(dl[i].x * An) * inv;
            bb.y = expm1f(dl[i].y * An) * inv;
            bu = mul2(mul2(Bv[i], bb), duv[i]);
          } else {
            bu = mul2(Bv[i], duv[i]);
          }
          // a_t h_{t-1} = h_t - b_t
          const float2 ah = add2(hv[i], make_float2(-bu.x, -bu.y));
          const float2 w = mul2(gv, ah);
          gA[i] = fma2(w, A2, gA[i]);
          dAl = fma2(w, dl[i], dAl);
          float2 db;
          if constexpr (kZOH) {
            // d b_t/d delta = a_t B u, d b_t/d A = B u (delta a_t - b_bar) / A
            const float2 gBu = mul2(gv, mul2(Bv[i], duv[i]));
            gA[i] = fma2(gBu, ab[i], gA[i]);
            const float inv = 1.f / An;
            dAl.x += gBu.x * (dl[i].x * ab[i].x - bb.x) * inv;
            dAl.y += gBu.y * (dl[i].y * ab[i].y - bb.y) * inv;
            gB[i] = fma2(gv, mul2(Bv[i], bb), gB[i]);
            db = mul2(gv, mul2(bb, duv[i]));
          } else {
            gB[i] = fma2(gv, Bv[i], gB[i]);
            db = mul2(gv, duv[i]);
          }
          if (i & 1) {
            db_hi = db;
          } else {
            float4& slot = tileB[tile_slot(lane * (kItems / 4) + (i >> 1))];
            const float4 v = slot;
            const float2 lo = add2(make_float2(v.x, v.y), db);
            const float2 hi = add2(make_float2(v.z, v.w), db_hi);
            slot = make_float4(lo.x, lo.y, hi.x, hi.y);
          }
        }
      }
      const float gnext = __shfl_sync(0xffffffffu, ab[0].x * g, 0);
      if (lane == 0) sh.gcarry[warp][n] = gnext;
      sh.dA[warp][n][lane] += dAl.x + dAl.y;
      if ((s + 1) % kPhase == 0) __syncthreads();
    }

    // ---- flush the dB/dC tiles of this chunk into global fp32 accumulators
    {
      const size_t base = static_cast<size_t>(b) * NS * L;
      for (int q = threadIdx.x; q < NS * (kChunk / 4); q += blockDim.x) {
        const int n = q / (kChunk / 4);
        const int qq = q % (kChunk / 4);
        const int slot = tile_slot(qq);
        float4 vb = make_float4(0.f, 0.f, 0.f, 0.f), vc = vb;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const float4 xb = sh.accB[r][n][slot];
          const float4 xc = sh.accC[r][n][slot];
          vb.x += xb.x; vb.y += xb.y; vb.z += xb.z; vb.w += xb.w;
          vc.x += xc.x; vc.y += xc.y; vc.z += xc.z; vc.w += xc.w;
          sh.accB[r][n][slot] = make_float4(0.f, 0.f, 0.f, 0.f);
          sh.accC[r][n][slot] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const int t = t0 + qq * 4;
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

    // ---- per-step epilogue
    if (active) {
      float2 uv[kHalf], dv[kHalf];
      load_run2(u_row, tl, lim, uv);
      load_run2(dl_row, tl, lim, dv);
      float2 o_du[kHalf], o_dd[kHalf];
#pragma unroll
      for (int i = 0; i < kHalf; ++i) {
        // ddelta_eff = sum_n g (B u + a h_{t-1} A)   (Euler; ZOH: gA holds all)
        float2 gd = kZOH ? gA[i] : fma2(uv[i], gB[i], gA[i]);
        if (p.delta_softplus) {
          gd.x *= sigmoid_f(dv[i].x + bias);
          gd.y *= sigmoid_f(dv[i].y + bias);
        }
        const float2 gu = kZOH ? gB[i] : mul2(dl[i], gB[i]);
        float2 du_ = fma2(dup2(Dv), dy[i], gu);
        const bool v0 = tl + 2 * i < lim, v1 = tl + 2 * i + 1 < lim;
        gd.x = v0 ? gd.x : 0.f;
        gd.y = v1 ? gd.y : 0.f;
        du_.x = v0 ? du_.x : 0.f;
        du_.y = v1 ? du_.y : 0.f;
        o_dd[i] = gd;
        o_du[i] = du_;
        dD_acc = fmaf(dy[i].x, uv[i].x, fmaf(dy[i].y, uv[i].y, dD_acc));
        dbias_acc += gd.x + gd.y;
      }
      store_run2(du_row, tl, L, o_du);
      store_run2(ddl_row, tl, L, o_dd);
      if (dz_row) {
        // dz = dout * (y + D u) * silu'(z), with y + D u saved by the forward
        float2 zv[kHalf], dov[kHalf], pv[kHalf], o_dz[kHalf];
        load_run2(z_row, tl, lim, zv);
        load_run2(dout_row, tl, lim, dov);
        load_run2(static_cast<const T*>(p.out_pre) + row * L, tl, lim, pv);
#pragma unroll
        for (int i = 0; i < kHalf; ++i) {
          const float s0 = sigmoid_f(zv[i].x), s1 = sigmoid_f(zv[i].y);
          o_dz[i].x = dov[i].x * pv[i].x * s0 * fmaf(zv[i].x, 1.f - s0, 1.f);
          o_dz[i].y = dov[i].y * pv[i].y * s1 * fmaf(zv[i].y, 1.f - s1, 1.f);
        }
        store_run2(dz_row, tl, L, o_dz);
      }
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
  const size_t smem = sizeof(BwdShared<NS>);
  auto kern = ss_bwd_kernel<NS, T, kZOH>;
  cudaError_t e = cudaFuncSetAttribute(
      kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  dim3 grid((p.dim + kBwdWarps - 1) / kBwdWarps, p.batch);
  kern<<<grid, kBwdWarps * 32, smem, stream>>>(p);
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

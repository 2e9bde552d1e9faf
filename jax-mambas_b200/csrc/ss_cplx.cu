// Complex selective scan (S6 with complex_ssm = True) for sm_100a.
//
// The reference evaluates this path in pure JAX (mamba/mamba1.py:170-176,
// 196): A (D, N), B, C (B, N, L) and the state complex, delta and u real,
//   a_t = exp(delta_t A),  b_t = delta_t B_t (Euler) or expm1(delta_t A) / A B_t,
//   h_t = a_t h_{t-1} + b_t u_t,   y_t = Re(C_t . h_t) + D u_t,
// with the fused softplus(delta + bias), padding mask and silu(z) gate of the
// real path. Gradients of complex arguments are dL/dRe + i dL/dIm (the
// adjoint G of the state obeys G_t = dy_t conj(C_t) + conj(a_{t+1}) G_{t+1}).
//
// Same decomposition as the real kernels (a lane owns up to 4 complex states
// of one channel, 8 channels per CTA, 32-step tiles; the forward saves the
// state after every 4 steps and the backward recomputes 4-step groups from
// those carries), with plain coalesced staging: this path is not the headline.
// exp(delta A) uses the accurate expf / sincosf: a slowly decaying complex
// mode sums the rounding of many steps.
#include <algorithm>

#include "ss_common.cuh"
#include "ss_launch.h"

namespace mss {

__device__ unsigned int g_cplx_device_error = 0;


template <int NS>
struct CplxCfg {
  static constexpr int kS = NS < 4 ? NS : 4;
  static constexpr int kLPC = NS / kS;
  static constexpr int kCPW = 32 / kLPC;
  static constexpr int kCh = kCPW < 8 ? 8 : kCPW;
  static constexpr int kWarps = kCh / kCPW;
  static constexpr int kThreads = kWarps * 32;
};

// (cos x, sin x) to about one ulp for |x| up to 2^20, in straight-line code
// (no large-argument path): Cody-Waite reduction x = k pi/2 + r, |r| <= pi/4,
// with pi/2 split into three floats (P1 + P2 + P3, each the float nearest the
// remainder) applied by fused multiply-adds, then the Taylor series of sin and
// cos about 0 through r^9 and r^10 (truncation below 1e-9 on |r| <= pi/4), and
// the quadrant k mod 4 choosing signs and order. The state of a slowly
// decaying complex mode accumulates the rounding of every step, so the SFU's
// approximate sin/cos are not used.
__device__ __forceinline__ float2 cis(float x) {
  constexpr float kTwoOverPi = 0x1.45f306p-1f;
  constexpr float kP1 = 0x1.921fb6p+0f, kP2 = -0x1.777a5cp-25f, kP3 = -0x1.ee59dap-50f;
  const float kf = rintf(x * kTwoOverPi);
  float r = fmaf(-kf, kP1, x);
  r = fmaf(-kf, kP2, r);
  r = fmaf(-kf, kP3, r);
  const int k = static_cast<int>(kf);
  const float r2 = r * r;
  // sin r = r (1 - r^2/3! + r^4/5! - r^6/7! + r^8/9!)
  float ps = fmaf(r2, 1.f / 362880.f, -1.f / 5040.f);
  ps = fmaf(ps, r2, 1.f / 120.f);
  ps = fmaf(ps, r2, -1.f / 6.f);
  const float sr = fmaf(ps * r2, r, r);
  // cos r = 1 - r^2/2! + r^4/4! - r^6/6! + r^8/8! - r^10/10!
  float pc = fmaf(r2, -1.f / 3628800.f, 1.f / 40320.f);
  pc = fmaf(pc, r2, -1.f / 720.f);
  pc = fmaf(pc, r2, 1.f / 24.f);
  pc = fmaf(pc, r2, -0.5f);
  const float cr = fmaf(pc, r2, 1.f);
  // quadrant: (cos, sin) of k pi/2 + r
  const bool swap = (k & 1) != 0;
  float c = swap ? sr : cr, sn = swap ? cr : sr;
  if (((k + 1) & 2) != 0) c = -c;
  if ((k & 2) != 0) sn = -sn;
  return make_float2(c, sn);
}

// cis() for two arguments at once: the same reduction and series with
// packed fp32x2 arithmetic (the quadrant logic per component). Returns
// (cos x.x, cos x.y) in c and (sin x.x, sin x.y) in s.
__device__ __forceinline__ void cis2(float2 x, float2& c, float2& s) {
  constexpr float kTwoOverPi = 0x1.45f306p-1f;
  constexpr float kP1 = 0x1.921fb6p+0f, kP2 = -0x1.777a5cp-25f, kP3 = -0x1.ee59dap-50f;
  const float2 q = mul2(x, dup2(kTwoOverPi));
  const float2 kf = make_float2(rintf(q.x), rintf(q.y));
  const float2 nkf = make_float2(-kf.x, -kf.y);
  float2 r = fma2(nkf, dup2(kP1), x);
  r = fma2(nkf, dup2(kP2), r);
  r = fma2(nkf, dup2(kP3), r);
  const int k0 = static_cast<int>(kf.x), k1 = static_cast<int>(kf.y);
  const float2 r2 = mul2(r, r);
  float2 ps = fma2(r2, dup2(1.f / 362880.f), dup2(-1.f / 5040.f));
  ps = fma2(ps, r2, dup2(1.f / 120.f));
  ps = fma2(ps, r2, dup2(-1.f / 6.f));
  const float2 sr = fma2(mul2(ps, r2), r, r);
  float2 pc = fma2(r2, dup2(-1.f / 3628800.f), dup2(1.f / 40320.f));
  pc = fma2(pc, r2, dup2(-1.f / 720.f));
  pc = fma2(pc, r2, dup2(1.f / 24.f));
  pc = fma2(pc, r2, dup2(-0.5f));
  const float2 cr = fma2(pc, r2, dup2(1.f));
  auto quad = [](int k, float cv, float sv, float& co, float& so) {
    const bool swap = (k & 1) != 0;
    co = swap ? sv : cv;
    so = swap ? cv : sv;
    if (((k + 1) & 2) != 0) co = -co;
    if ((k & 2) != 0) so = -so;
  };
  quad(k0, cr.x, sr.x, c.x, s.x);
  quad(k1, cr.y, sr.y, c.y, s.y);
}

struct Cx {
  float r, i;
};
__device__ __forceinline__ Cx cmul(Cx a, Cx b) { return {a.r * b.r - a.i * b.i, a.r * b.i + a.i * b.r}; }
__device__ __forceinline__ Cx cmulc(Cx a, Cx b) {  // a * conj(b)
  return {a.r * b.r + a.i * b.i, a.i * b.r - a.r * b.i};
}
__device__ __forceinline__ Cx cconj(Cx a) { return {a.r, -a.i}; }
__device__ __forceinline__ Cx cld(const float2* p) { const float2 v = *p; return {v.x, v.y}; }

// Euler discretization of two states at one step: a_j = exp(delta A_j) =
// 2^(delta Re A_j log2 e) cis(delta Im A_j), the modulus from the SFU's ex2
// (as the real kernels' decay), the rotation from cis2.
__device__ __forceinline__ void cdisc_euler2(float dl, Cx A0, Cx A1, Cx& a0, Cx& a1) {
  float2 c, sn;
  cis2(mul2(dup2(dl), make_float2(A0.i, A1.i)), c, sn);
  const float2 arg = mul2(dup2(dl * kLog2e), make_float2(A0.r, A1.r));
  const float m0 = ex2(arg.x), m1 = ex2(arg.y);
  const float2 re = mul2(make_float2(m0, m1), c), im = mul2(make_float2(m0, m1), sn);
  a0 = {re.x, im.x};
  a1 = {re.y, im.y};
}

// a = exp(delta A) and (ZOH) bb = expm1(delta A) / A, for complex A = (ar, ai)
template <bool kZOH>
__device__ __forceinline__ void cdisc(float dl, Cx A, Cx& a, Cx& bb) {
  const float2 cs = cis(dl * A.i);
  const float m = expf(dl * A.r);
  a = {m * cs.x, m * cs.y};
  if constexpr (kZOH) {
    // expm1(x + iy) = expm1(x) cos y - 2 sin^2(y/2) + i e^x sin y, over A
    const float sh = cis(0.5f * dl * A.i).y;
    const Cx e1 = {fmaf(expm1f(dl * A.r), cs.x, -2.f * sh * sh), m * cs.y};
    const float den = A.r * A.r + A.i * A.i;
    bb = {(e1.r * A.r + e1.i * A.i) / den, (e1.i * A.r - e1.r * A.i) / den};
  } else {
    bb = {dl, 0.f};
  }
}


// The forward's staging: tiles of kFT steps; delta, u, z and B, C of the next
// tile are copied in by cp.async (zero-filled past the valid length) while
// the current tile is scanned.
constexpr int kFT = 16;
constexpr int kFRow = kFT + 4;
template <int kCh>
struct CplxFwdShared {
  float dlt[kCh][kFRow];  // delta_eff
  float uu[kCh][kFRow];   // u (masked)
  float yy[kCh][kFRow];   // D u, then + y
  float rD[2][kCh][kFT];  // raw delta, u, z (two buffers)
  float rU[2][kCh][kFT];
  float rZ[2][kCh][kFT];
  float2 Bt[2][16][kFT];
  float2 Ct[2][16][kFT];
};

template <int NS, bool kZOH>
__global__ void __launch_bounds__(CplxCfg<NS>::kThreads)
    ss_cfwd_kernel(const CplxParams p) {
  using Cfg = CplxCfg<NS>;
  constexpr int kS = Cfg::kS, kLPC = Cfg::kLPC, kCh = Cfg::kCh, kThreads = Cfg::kThreads;
  constexpr int kCT = kFT;
  __shared__ CplxFwdShared<kCh> sh;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.y, d0 = blockIdx.x * kCh;
  const int L = p.seqlen;
  const int n_ch = min(kCh, p.dim - d0);
  const int cl = warp * Cfg::kCPW + lane / kLPC;
  const int q = lane % kLPC;
  const bool act = cl < n_ch;
  const int d = d0 + (act ? cl : 0);
  const size_t row = static_cast<size_t>(b) * p.dim + d;
  int len = L;
  if (p.seq_lens) len = max(0, min(L, p.seq_lens[b]));
  const float2* A2 = static_cast<const float2*>(p.A);
  const float2* B2 = static_cast<const float2*>(p.B) + static_cast<size_t>(b) * NS * L;
  const float2* C2 = static_cast<const float2*>(p.C) + static_cast<size_t>(b) * NS * L;
  Cx Av[kS], h[kS];
#pragma unroll
  for (int j = 0; j < kS; ++j) {
    const int n = q + kLPC * j;
    Av[j] = cld(A2 + d * NS + n);
    h[j] = {0.f, 0.f};
    if (act && p.h0) h[j] = cld(static_cast<const float2*>(p.h0) + row * NS + n);
  }
  const size_t bdl = static_cast<size_t>(b) * p.dim * L;
  const float* zb = p.z ? p.z : p.u;  // a valid address when z is absent
  // ---- staging of tile t0s into buffer sb (asynchronous, one commit group)
  auto stage = [&](int t0s, int sb) {
    for (int i = tid; i < kCh * kCT; i += kThreads) {
      const int c = i / kCT, tt = i % kCT, t = t0s + tt;
      const bool v = c < n_ch && t < len;
      const size_t off = v ? bdl + static_cast<size_t>(d0 + c) * L + t : 0;
      cp_async4(&sh.rD[sb][c][tt], p.delta + off, v);
      cp_async4(&sh.rU[sb][c][tt], p.u + off, v);
      cp_async4(&sh.rZ[sb][c][tt], zb + off, v && p.z != nullptr);
    }
    for (int i = tid; i < NS * kCT; i += kThreads) {
      const int n = i / kCT, tt = i % kCT, t = t0s + tt;
      const bool v = t < len;
      const size_t off = v ? static_cast<size_t>(n) * L + t : 0;
      cp_async8(&sh.Bt[sb][n][tt], B2 + off, v);
      cp_async8(&sh.Ct[sb][n][tt], C2 + off, v);
    }
    cp_async_commit();
  };
  stage(0, 0);
  for (int t0 = 0; t0 < L; t0 += kCT) {
    const int sb = (t0 / kCT) & 1;
    // the next tile's copies fly while this one is scanned (an empty group
    // past the end keeps the wait below uniform)
    if (t0 + kCT < L) {
      stage(t0 + kCT, sb ^ 1);
    } else {
      cp_async_commit();
    }
    cp_async_wait<1>();
    __syncthreads();
    // ---- transform: delta_eff, u, D u (rows)
    for (int i = tid; i < kCh * kCT; i += kThreads) {
      const int c = i / kCT, tt = i % kCT, t = t0 + tt;
      float dv = 0.f, uv = 0.f, yd = 0.f;
      if (c < n_ch && t < len) {
        const float x = sh.rD[sb][c][tt] + (p.delta_bias ? p.delta_bias[d0 + c] : 0.f);
        dv = p.delta_softplus ? softplus_f(x) : x;
        uv = sh.rU[sb][c][tt];
        yd = p.D ? p.D[d0 + c] * uv : 0.f;
      }
      sh.dlt[c][tt] = dv;
      sh.uu[c][tt] = uv;
      sh.yy[c][tt] = yd;
    }
    __syncthreads();
    // ---- scan, one step per iteration (rolled: the per-step body is long);
    // steps past the valid length carry delta = 0 and leave the state as is
    const int steps4 = (min(kCT, len - t0) + 3) & ~3;
#pragma unroll 1
    for (int tt = 0; tt < steps4; ++tt) {
      const float dl = sh.dlt[cl][tt];
      const float uv = sh.uu[cl][tt];
      const float dlu = dl * uv;
      float yp = 0.f;
      Cx av[kS], bbs[kS];
#pragma unroll
      for (int j = 0; j < kS; ++j) {
        if (!kZOH && (j & 1) == 0 && j + 1 < kS) {
          cdisc_euler2(dl, Av[j], Av[j + 1], av[j], av[j + 1]);
          bbs[j] = bbs[j + 1] = {dl, 0.f};
        } else if (kZOH || (j & 1) == 0) {
          cdisc<kZOH>(dl, Av[j], av[j], bbs[j]);
        }
      }
#pragma unroll
      for (int j = 0; j < kS; ++j) {
        const int n = q + kLPC * j;
        const Cx a = av[j], bb = bbs[j];
        const Cx Bn = cld(&sh.Bt[sb][n][tt]);
        // Euler: b_bar u = delta u B (real times complex)
        const Cx bu = kZOH ? cmul(bb, {Bn.r * uv, Bn.i * uv}) : Cx{dlu * Bn.r, dlu * Bn.i};
        h[j] = {fmaf(a.r, h[j].r, fmaf(-a.i, h[j].i, bu.r)),
                fmaf(a.r, h[j].i, fmaf(a.i, h[j].r, bu.i))};
        const Cx Cn = cld(&sh.Ct[sb][n][tt]);
        yp = fmaf(Cn.r, h[j].r, fmaf(-Cn.i, h[j].i, yp));
      }
#pragma unroll
      for (int m = 1; m < kLPC; m <<= 1) yp += __shfl_xor_sync(0xffffffffu, yp, m);
      if (q == 0) sh.yy[cl][tt] += yp;
      if (act && (tt & 3) == 3) {  // carry after each 4 steps, natural state order
        float2* cs = static_cast<float2*>(p.chunk_states) +
                     carry_offset(b, (t0 + tt) / kCkpt, p.n_chunks, p.dim, d, NS);
#pragma unroll
        for (int j = 0; j < kS; ++j) cs[q + kLPC * j] = make_float2(h[j].r, h[j].i);
      }
    }
    __syncthreads();
    // ---- emit
    for (int i = tid; i < kCh * kCT; i += kThreads) {
      const int c = i / kCT, tt = i % kCT, t = t0 + tt;
      if (c >= n_ch || t >= L) continue;
      const size_t off = bdl + static_cast<size_t>(d0 + c) * L + t;
      float pre = 0.f, o = 0.f;
      if (t < len) {
        pre = sh.yy[c][tt];
        o = p.z ? pre * silu_f(sh.rZ[sb][c][tt]) : pre;
      }
      p.out[off] = o;
      if (p.out_pre) p.out_pre[off] = pre;
    }
    __syncthreads();
  }
  if (p.last_state && act) {
#pragma unroll
    for (int j = 0; j < kS; ++j)
      static_cast<float2*>(p.last_state)[row * NS + q + kLPC * j] = make_float2(h[j].r, h[j].i);
  }
}

// The backward's staging: tiles of kGT steps (two groups); delta, u, dout,
// z, the pre-gate output and B, C of the next tile (to the left) are copied
// in by cp.async while the current one is processed. Short tiles keep the
// double buffers within the shared memory that lets 11 one-warp CTAs reside
// per SM (a configs[1] layer's whole grid in one wave).
constexpr int kGT = 8;
constexpr int kGRow = kGT + 4;
template <int kCh>
struct CplxBwdShared {
  float dlt[kCh][kGRow];  // delta_eff
  float uu[kCh][kGRow];   // u (masked)
  float yy[kCh][kGRow];   // dy
  float rD[2][kCh][kGT];  // raw delta, u, dout, z, pre-gate (two buffers)
  float rU[2][kCh][kGT];
  float rY[2][kCh][kGT];
  float rZ[2][kCh][kGT];
  float rP[2][kCh][kGT];
  float2 Bt[2][16][kGT];
  float2 Ct[2][16][kGT];
};

template <int NS, bool kZOH>
__global__ void __launch_bounds__(CplxCfg<NS>::kThreads, CplxCfg<NS>::kThreads == 32 ? 11 : 1)
    ss_cbwd_kernel(const CplxParams p) {
  using Cfg = CplxCfg<NS>;
  constexpr int kS = Cfg::kS, kLPC = Cfg::kLPC, kCh = Cfg::kCh, kThreads = Cfg::kThreads;
  constexpr int kCT = kGT;
  static_assert(Cfg::kWarps == 1, "the channel sums of dB / dC are per warp");
  __shared__ CplxBwdShared<kCh> sh;
  // one group's dB (re, im) and dC (re, im) per (channel, swizzled state),
  // summed over the warp's channels by flush_part
  __shared__ float4 part[4][kCh][NS];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.y, d0 = blockIdx.x * kCh;
  const int L = p.seqlen;
  const int n_ch = min(kCh, p.dim - d0);
  const int cl = warp * Cfg::kCPW + lane / kLPC;
  const int q = lane % kLPC;
  const bool act = cl < n_ch;
  const int d = d0 + (act ? cl : 0);
  const size_t row = static_cast<size_t>(b) * p.dim + d;
  int len = L;
  if (p.seq_lens) len = max(0, min(L, p.seq_lens[b]));
  const float2* A2 = static_cast<const float2*>(p.A);
  const float2* B2 = static_cast<const float2*>(p.B) + static_cast<size_t>(b) * NS * L;
  const float2* C2 = static_cast<const float2*>(p.C) + static_cast<size_t>(b) * NS * L;
  const float Dv = p.D ? p.D[d] : 0.f;
  Cx Av[kS], Gp[kS];
  float dAr[kS], dAi[kS];
#pragma unroll
  for (int j = 0; j < kS; ++j) {
    const int n = q + kLPC * j;
    Av[j] = cld(A2 + d * NS + n);
    // conj(a_{t+1}) G_{t+1} of the step after the current one: dlast at the end
    Gp[j] = {0.f, 0.f};
    if (act && p.dlast) Gp[j] = cld(static_cast<const float2*>(p.dlast) + row * NS + n);
    dAr[j] = dAi[j] = 0.f;
  }
  float dD_acc = 0.f, dbias_acc = 0.f;
  const size_t bdl = static_cast<size_t>(b) * p.dim * L;
  const int n_tiles = len > 0 ? (len - 1) / kCT + 1 : 0;
  // steps at or past the valid length: zero gradients (the groups below skip
  // them)
  for (int i = tid; i < kCh * L; i += kThreads) {
    const int c = i / L, t = i % L;
    if (c < n_ch && t >= len) {
      const size_t off = bdl + static_cast<size_t>(d0 + c) * L + t;
      p.du[off] = 0.f;
      p.ddelta[off] = 0.f;
      if (p.dz) p.dz[off] = 0.f;
    }
  }
  const float* zb = p.z ? p.z : p.u;  // valid addresses when z is absent
  const float* pb = p.out_pre ? p.out_pre : p.u;
  // ---- staging of tile t0s into buffer sb (asynchronous, one commit group)
  auto stage = [&](int t0s, int sb) {
    for (int i = tid; i < kCh * kCT; i += kThreads) {
      const int c = i / kCT, tt = i % kCT, t = t0s + tt;
      const bool v = c < n_ch && t < len;
      const size_t off = v ? bdl + static_cast<size_t>(d0 + c) * L + t : 0;
      cp_async4(&sh.rD[sb][c][tt], p.delta + off, v);
      cp_async4(&sh.rU[sb][c][tt], p.u + off, v);
      cp_async4(&sh.rY[sb][c][tt], p.dout + off, v);
      cp_async4(&sh.rZ[sb][c][tt], zb + off, v && p.z != nullptr);
      cp_async4(&sh.rP[sb][c][tt], pb + off, v && p.z != nullptr);
    }
    for (int i = tid; i < NS * kCT; i += kThreads) {
      const int n = i / kCT, tt = i % kCT, t = t0s + tt;
      const bool v = t < len;
      const size_t off = v ? static_cast<size_t>(n) * L + t : 0;
      cp_async8(&sh.Bt[sb][n][tt], B2 + off, v);
      cp_async8(&sh.Ct[sb][n][tt], C2 + off, v);
    }
    cp_async_commit();
  };
  // the state entering group gi (saved carry, or h0)
  auto load_hs = [&](int gi, Cx (&hs)[kS]) {
#pragma unroll
    for (int j = 0; j < kS; ++j) {
      const int n = q + kLPC * j;
      hs[j] = {0.f, 0.f};
      if (act) {
        if (gi > 0)
          hs[j] = cld(static_cast<const float2*>(p.chunk_states) +
                      carry_offset(b, gi - 1, p.n_chunks, p.dim, d, NS) + n);
        else if (p.h0)
          hs[j] = cld(static_cast<const float2*>(p.h0) + row * NS + n);
      }
    }
  };
  if (n_tiles > 0) stage((n_tiles - 1) * kCT, 0);
  for (int k = n_tiles - 1; k >= 0; --k) {
    const int t0 = k * kCT;
    const int sb = (n_tiles - 1 - k) & 1;
    __syncthreads();  // every thread is done with buffer sb ^ 1 (the previous tile's)
    if (k > 0) {
      stage(t0 - kCT, sb ^ 1);
    } else {
      cp_async_commit();
    }
    // the carry entering the tile's last valid group, loaded while the copies land
    const int g_first = min(kCT / 4 - 1, (len - 1 - t0) / 4);
    Cx hs_next[kS];
    load_hs((t0 + g_first * 4) / kCkpt, hs_next);
    cp_async_wait<1>();
    __syncthreads();
    // ---- transform: delta_eff, u, dy; dz written directly
    for (int i = tid; i < kCh * kCT; i += kThreads) {
      const int c = i / kCT, tt = i % kCT, t = t0 + tt;
      float dv = 0.f, uv = 0.f, dy = 0.f;
      if (c < n_ch && t < L) {
        const size_t off = bdl + static_cast<size_t>(d0 + c) * L + t;
        float dz = 0.f;
        if (t < len) {
          float x = sh.rD[sb][c][tt] + (p.delta_bias ? p.delta_bias[d0 + c] : 0.f);
          dv = p.delta_softplus ? softplus_f(x) : x;
          uv = sh.rU[sb][c][tt];
          dy = sh.rY[sb][c][tt];
          if (p.z) {
            const float zv = sh.rZ[sb][c][tt], sz = sigmoid_f(zv);
            dz = dy * sh.rP[sb][c][tt] * sz * fmaf(zv, 1.f - sz, 1.f);
            dy *= zv * sz;
          }
        }
        if (p.dz) p.dz[off] = dz;
      }
      sh.dlt[c][tt] = dv;
      sh.uu[c][tt] = uv;
      sh.yy[c][tt] = dy;
    }
    __syncthreads();
    // ---- groups of 4 steps in reverse
    for (int g = g_first; g >= 0; --g) {
      const int tg = g * 4;
      Cx hs[kS];
#pragma unroll
      for (int j = 0; j < kS; ++j) hs[j] = hs_next[j];
      if (g > 0) load_hs((t0 + tg - 4) / kCkpt, hs_next);
      // recompute a, bb, h over the group (h[e][j] = state after step e)
      Cx aa[4][kS], bbv[4][kS], hh[5][kS];
#pragma unroll
      for (int j = 0; j < kS; ++j) hh[0][j] = hs[j];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float dl = sh.dlt[cl][tg + e], uv = sh.uu[cl][tg + e];
        const float dlu = dl * uv;
#pragma unroll
        for (int j = 0; j < kS; ++j) {
          if (!kZOH && (j & 1) == 0 && j + 1 < kS) {
            cdisc_euler2(dl, Av[j], Av[j + 1], aa[e][j], aa[e][j + 1]);
            bbv[e][j] = bbv[e][j + 1] = {dl, 0.f};
          } else if (kZOH || (j & 1) == 0) {
            cdisc<kZOH>(dl, Av[j], aa[e][j], bbv[e][j]);
          }
        }
#pragma unroll
        for (int j = 0; j < kS; ++j) {
          const int n = q + kLPC * j;
          const Cx Bn = cld(&sh.Bt[sb][n][tg + e]);
          const Cx bu =
              kZOH ? cmul(bbv[e][j], {Bn.r * uv, Bn.i * uv}) : Cx{dlu * Bn.r, dlu * Bn.i};
          const Cx& a = aa[e][j];
          const Cx& hp = hh[e][j];
          hh[e + 1][j] = {fmaf(a.r, hp.r, fmaf(-a.i, hp.i, bu.r)),
                          fmaf(a.r, hp.i, fmaf(a.i, hp.r, bu.i))};
        }
      }
      float sB[4], sA[4];  // per step: sum_n Re(G conj(B)) (ZOH: Re(G conj(bb B))), sum_n Re(G conj(h) conj(A a))
      // (Euler ddelta's b-part is u * sB; ZOH's is in sA)
#pragma unroll
      for (int e = 3; e >= 0; --e) {
        const float dl = sh.dlt[cl][tg + e], uv = sh.uu[cl][tg + e], dy = sh.yy[cl][tg + e];
        sB[e] = sA[e] = 0.f;
#pragma unroll
        for (int j = 0; j < kS; ++j) {
          const int n = q + kLPC * j;
          const Cx Cn = cld(&sh.Ct[sb][n][tg + e]);
          const Cx Bn = cld(&sh.Bt[sb][n][tg + e]);
          // G_t = dy conj(C_t) + conj(a_{t+1}) G_{t+1}
          const Cx Gt = {fmaf(dy, Cn.r, Gp[j].r), fmaf(-dy, Cn.i, Gp[j].i)};
          const Cx& a = aa[e][j];
          const Cx& hp = hh[e][j];
          // dC = dy conj(h_t), dB = G conj(bb) u
          const Cx ht = hh[e + 1][j];
          const Cx dCv = {dy * ht.r, -dy * ht.i};
          // Euler: G conj(bb) u = G delta u
          const Cx gbb = kZOH ? cmulc(Gt, bbv[e][j]) : Cx{Gt.r * dl, Gt.i * dl};
          const Cx dBv = {gbb.r * uv, gbb.i * uv};
          {
            const int col = n ^ part_swz<NS>(cl);
            reinterpret_cast<float*>(&part[0][cl][col])[e] = dBv.r;
            reinterpret_cast<float*>(&part[1][cl][col])[e] = dBv.i;
            reinterpret_cast<float*>(&part[2][cl][col])[e] = dCv.r;
            reinterpret_cast<float*>(&part[3][cl][col])[e] = dCv.i;
          }
          // Euler: Re(G conj(B)) (du = delta * sum, ddelta's b-part u * sum);
          // ZOH: Re(G conj(bb B)) (du = sum). ga = G conj(h_{t-1})
          const Cx gB = kZOH ? cmulc(Gt, cmul(bbv[e][j], Bn)) : cmulc(Gt, Bn);
          sB[e] += gB.r;
          const Cx ga = cmulc(Gt, hp);
          const Cx Aa = cmul(Av[j], a);
          sA[e] += cmulc(ga, Aa).r;
          const Cx dAv = cmulc(ga, a);  // times delta
          dAr[j] = fmaf(dl, dAv.r, dAr[j]);
          dAi[j] = fmaf(dl, dAv.i, dAi[j]);
          if constexpr (kZOH) {
            // bb = expm1(delta A) / A: dbb/ddelta = a, dbb/dA = (delta a - bb) / A
            const Cx gBu = cmulc(Gt, {Bn.r * uv, Bn.i * uv});
            sA[e] += cmulc(gBu, a).r;
            const Cx num = {dl * a.r - bbv[e][j].r, dl * a.i - bbv[e][j].i};
            const float den = Av[j].r * Av[j].r + Av[j].i * Av[j].i;
            const Cx dbdA = {(num.r * Av[j].r + num.i * Av[j].i) / den,
                             (num.i * Av[j].r - num.r * Av[j].i) / den};
            const Cx t2 = cmulc(gBu, dbdA);
            dAr[j] += t2.r;
            dAi[j] += t2.i;
          }
          Gp[j] = cmulc(Gt, a);  // conj(a_t) G_t, seen by step t - 1
        }
      }
      // dB, dC of the group: sums over the warp's channels into the planes
      __syncwarp();
      {
        const bool whole = t0 + tg + 4 <= len && (L & 3) == 0;
        const size_t bo = static_cast<size_t>(b) * NS * L;
        flush_part<NS>(part[0], p.dB_acc_r + bo, L, t0 + tg, len, whole, lane);
        flush_part<NS>(part[1], p.dB_acc_i + bo, L, t0 + tg, len, whole, lane);
        flush_part<NS>(part[2], p.dC_acc_r + bo, L, t0 + tg, len, whole, lane);
        flush_part<NS>(part[3], p.dC_acc_i + bo, L, t0 + tg, len, whole, lane);
      }
      __syncwarp();
      // sums over the channel's lanes, then du, ddelta
#pragma unroll
      for (int m = 1; m < kLPC; m <<= 1)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          sB[e] += __shfl_xor_sync(0xffffffffu, sB[e], m);
          sA[e] += __shfl_xor_sync(0xffffffffu, sA[e], m);
        }
      if (q == 0 && act) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = t0 + tg + e;
          if (t >= L) continue;
          const size_t off = bdl + static_cast<size_t>(d) * L + t;
          const float dl = sh.dlt[cl][tg + e], uv = sh.uu[cl][tg + e], dy = sh.yy[cl][tg + e];
          float gd = kZOH ? sA[e] : fmaf(uv, sB[e], sA[e]);
          if (p.delta_softplus) gd *= sigmoid_from_softplus(dl);
          const float du = fmaf(Dv, dy, kZOH ? sB[e] : dl * sB[e]);
          const bool valid = t < len;
          p.du[off] = valid ? du : 0.f;
          p.ddelta[off] = valid ? gd : 0.f;
          dbias_acc += valid ? gd : 0.f;
          dD_acc = fmaf(dy, uv, dD_acc);  // dy, u are 0 past the end
        }
      }
    }
  }
  // ---- per-row results: dA (complex) and dD / dbias partials, dh0
  if (act) {
#pragma unroll
    for (int j = 0; j < kS; ++j) {
      const int n = q + kLPC * j;
      p.dA_part[(row * NS + n) * 2] = dAr[j];
      p.dA_part[(row * NS + n) * 2 + 1] = dAi[j];
      if (p.dh0)
        static_cast<float2*>(p.dh0)[row * NS + n] = make_float2(Gp[j].r, Gp[j].i);
    }
    if (q == 0) {
      p.dD_part[row] = dD_acc;
      p.dbias_part[row] = dbias_acc;
    }
  }
}

// (re, im) planes -> interleaved complex64
__global__ void interleave_kernel(const float* __restrict__ re, const float* __restrict__ im,
                                  float2* out, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    out[i] = make_float2(re[i], im[i]);
}

template <int NS, bool kZOH>
static cudaError_t launch_cplx_t(const CplxParams& p, bool backward, cudaStream_t stream) {
  using Cfg = CplxCfg<NS>;
  dim3 grid((p.dim + Cfg::kCh - 1) / Cfg::kCh, p.batch);
  if (backward)
    ss_cbwd_kernel<NS, kZOH><<<grid, Cfg::kThreads, 0, stream>>>(p);
  else
    ss_cfwd_kernel<NS, kZOH><<<grid, Cfg::kThreads, 0, stream>>>(p);
  return cudaPeekAtLastError();
}

template <bool kZOH>
static cudaError_t launch_cplx_n(const CplxParams& p, int dstate, bool backward,
                                 cudaStream_t stream) {
  switch (dstate) {
    case 1: return launch_cplx_t<1, kZOH>(p, backward, stream);
    case 2: return launch_cplx_t<2, kZOH>(p, backward, stream);
    case 4: return launch_cplx_t<4, kZOH>(p, backward, stream);
    case 8: return launch_cplx_t<8, kZOH>(p, backward, stream);
    case 16: return launch_cplx_t<16, kZOH>(p, backward, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_cplx_fwd(const CplxParams& p, int dstate, int zoh, cudaStream_t stream) {
  return zoh ? launch_cplx_n<true>(p, dstate, false, stream)
             : launch_cplx_n<false>(p, dstate, false, stream);
}

cudaError_t launch_cplx_bwd(const CplxParams& p, int dstate, int zoh, void* dA, void* dB,
                            void* dC, float* dD, float* ddelta_bias, cudaStream_t stream) {
  const size_t n_bnl = static_cast<size_t>(p.batch) * dstate * p.seqlen;
  for (float* acc : {p.dB_acc_r, p.dB_acc_i, p.dC_acc_r, p.dC_acc_i}) {
    cudaError_t e = cudaMemsetAsync(acc, 0, n_bnl * sizeof(float), stream);
    if (e != cudaSuccess) return e;
  }
  cudaError_t e = zoh ? launch_cplx_n<true>(p, dstate, true, stream)
                      : launch_cplx_n<false>(p, dstate, true, stream);
  if (e != cudaSuccess) return e;
  // dA (complex, as 2 dstate real columns), dD, ddelta_bias: fixed-order batch sums
  e = launch_param_reduce(p.dA_part, p.dD_part, p.dbias_part, static_cast<float*>(dA), dD,
                          ddelta_bias, p.batch, p.dim, 2 * dstate, stream);
  if (e != cudaSuccess) return e;
  const int blocks = static_cast<int>(std::min<size_t>((n_bnl + 255) / 256, 148 * 16));
  interleave_kernel<<<blocks, 256, 0, stream>>>(p.dB_acc_r, p.dB_acc_i, static_cast<float2*>(dB),
                                                 n_bnl);
  interleave_kernel<<<blocks, 256, 0, stream>>>(p.dC_acc_r, p.dC_acc_i, static_cast<float2*>(dC),
                                                 n_bnl);
  return cudaPeekAtLastError();
}

}  // namespace mss

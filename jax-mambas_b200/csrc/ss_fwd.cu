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
// kCh channels of one batch (one warp for N = 16, so that every CTA of a
// Mamba-size layer is resident at once). The CTA walks L in tiles of kTile
// steps, double-buffered:
//   0. TMA: one thread issues five 2-D tensor copies per tile (delta, u, z as
//      [kCh channels x kTile steps], B, C as [N states x kTile steps]) into a
//      staging buffer, completing on an mbarrier; the TMA zero-fills past the
//      sequence end and past the last channel; the next tile's copies fly
//      while this tile computes;
//   1. transform: delta_eff = softplus(delta + bias) and delta_eff*u are
//      formed once per element into fp32 work tiles, B and C are widened;
//   2. scan: each lane steps through the tile; per step and state one
//      2^(delta*A*log2 e) on the SFU and packed fp32x2 multiply-adds, then the
//      kS-state partial sums of C_t h_t are reduced over the channel's lanes;
//   3. emit: out = (y + D u) * silu(z) and the pre-gate y + D u (read by the
//      backward for dz) are written coalesced.
// The state after every MSS_CHUNK (4) steps is saved for the backward. Rows whose
// length or base address is not 16-byte aligned take the same path with the
// staging done by plain loads instead of TMA.
#include <cudaTypedefs.h>

#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <type_traits>

#include "ss_common.cuh"
#include "ss_launch.h"

namespace mss {

__device__ unsigned int g_fwd_device_error = 0;

constexpr int kTile = 32;  // steps staged per pass
constexpr int kPad = 4;    // row padding (floats) of the fp32 work tiles
constexpr int kRow = kTile + kPad;
static_assert(kTile % kCkpt == 0 && kCkpt == 4, "a carry is saved after every 4 steps");

// kWide: four warps per CTA share one B/C staging (N = 16 only; chosen for
// grids of several waves, where the smaller shared-memory share per warp
// lets more warps reside per SM)
template <int NS, bool kWide = false>
struct FwdCfg {
  static constexpr int kS = NS < 4 ? NS : 4;  // states per lane
  static constexpr int kLPC = NS / kS;        // lanes per channel
  static constexpr int kCPW = 32 / kLPC;      // channels per warp
  static constexpr int kCh = kWide ? 4 * kCPW : (kCPW < 8 ? 8 : kCPW);  // channels per CTA
  static constexpr int kWarps = kCh / kCPW;   // warps per CTA
  static constexpr int kThreads = kWarps * 32;
};

// Tensor maps of the five TMA-staged inputs (see launch_fwd).
struct FwdMaps {
  CUtensorMap d, u, z, b, c;
};

template <int NS, typename T, bool kWide = false>
struct FwdShared {
  static constexpr int kCh = FwdCfg<NS, kWide>::kCh;
  // staging, written by TMA (two buffers); every block is a multiple of 128 B
  alignas(128) T rawD[2][kCh][kTile];
  T rawU[2][kCh][kTile];
  T rawZ[2][kCh][kTile];
  // B/C blocks padded to whole 1024-byte units: fp32 B/C are staged with the
  // TMA's 128-byte swizzle, whose pattern repeats every 8 rows of 128 bytes.
  static constexpr int kNSP =
      (NS * kTile * sizeof(T) + 1023) / 1024 * 1024 / (kTile * sizeof(T));
  alignas(1024) T rawB[2][kNSP][kTile];
  alignas(1024) T rawC[2][kNSP][kTile];
  // fp32 work tiles
  float dlt[kCh][kRow];  // delta_eff
  // delta_eff * u (ZOH: u); each 4-step group's entries are overwritten by
  // y_t = sum_n C_t h_t of those steps once every lane has read them
  float dlu[kCh][kRow];
  // widened B/C (bf16 I/O only; fp32 I/O reads the swizzled staging)
  float Bs[sizeof(T) == 4 ? 1 : NS][kRow];
  float Cs[sizeof(T) == 4 ? 1 : NS][kRow];
  uint64_t bar[2];
};

// Four consecutive staged elements as fp32 (16-byte or 8-byte aligned).
__device__ __forceinline__ void load4_smem(const float* src, float (&v)[4]) {
  const float4 f = *reinterpret_cast<const float4*>(src);
  v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
}
__device__ __forceinline__ void load4_smem(const __nv_bfloat16* src, float (&v)[4]) {
  const float4 f = bf16x4_to_f32(*reinterpret_cast<const uint2*>(src));
  v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
}
__device__ __forceinline__ void store4_global(float* dst, const float (&v)[4]) {
  *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void store4_global(__nv_bfloat16* dst, const float (&v)[4]) {
  uint2 w;
  *reinterpret_cast<__nv_bfloat162*>(&w.x) = __floats2bfloat162_rn(v[0], v[1]);
  *reinterpret_cast<__nv_bfloat162*>(&w.y) = __floats2bfloat162_rn(v[2], v[3]);
  *reinterpret_cast<uint2*>(dst) = w;
}

// kEnd: the end-state pass of a segmented scan (no outputs; each segment from
// a zero state, its final state and sum of delta_eff to seg_end / seg_dsum).
// kLPT: right-padded batches, grid rows take the sequences longest first
// (batch_of_row).
// kStd: the fused layer's usual call (softplus on delta, a z gate, the
// pre-gate output and the carries saved for the backward), with those
// choices compiled in instead of tested per element or step group.
template <int NS, typename T, bool kZOH, bool kEnd, bool kWide, bool kLPT = false,
          bool kStd = false>
__global__ void __launch_bounds__(FwdCfg<NS, kWide>::kThreads)
    ss_fwd_kernel(const FwdParams p, const __grid_constant__ FwdMaps maps) {
  using Cfg = FwdCfg<NS, kWide>;
  constexpr int kS = Cfg::kS;
  constexpr int kLPC = Cfg::kLPC;
  constexpr int kCh = Cfg::kCh;
  constexpr int kThreads = Cfg::kThreads;
  // fp32 B/C are read straight from the (swizzled) TMA staging; B/C rows past
  // the sequence end are zero-filled by the TMA, and their steps carry
  // delta = 0, so they never touch the state.
  constexpr bool kDirectBC = sizeof(T) == 4;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  using Sh = FwdShared<NS, T, kWide>;
  Sh& sh = *reinterpret_cast<Sh*>(smem_raw);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int b = kLPT ? batch_of_row(p.seq_lens, p.batch, p.seqlen, static_cast<int>(blockIdx.y))
                     : static_cast<int>(blockIdx.y);
  const int d0 = blockIdx.x * kCh;
  const int L = p.seqlen;
  const int n_ch = min(kCh, p.dim - d0);  // live channels of this CTA

  // this lane's channel slot and states: slot j holds state
  // q + kLPC (j ^ perm) (a permutation of q, q + kLPC, ...; see state_perm)
  const int cl = warp * Cfg::kCPW + lane / kLPC;
  const int q = lane % kLPC;
  const int perm = state_perm<NS>(cl);
  auto st_of = [&](int j) { return q + kLPC * (j ^ perm); };
  const bool lane_active = cl < n_ch;
  const int d = d0 + (lane_active ? cl : 0);
  const size_t row = static_cast<size_t>(b) * p.dim + d;

  int len = L;
  if (p.seq_lens MSS_AND(in_bounds(b, p.batch, kSiteSeqLens)))
    len = max(0, min(L, p.seq_lens[b]));
  // extents of the arrays, in elements (bounds build only)
  MSS_BOUNDS_ONLY(const long long n_bd = static_cast<long long>(p.batch) * p.dim;
                  const long long n_rows = n_bd * L;
                  const long long n_bc = static_cast<long long>(p.batch) * NS * L;)

  // this CTA's time segment: tiles [k_begin, k_end)
  const int seg = blockIdx.z;
  const int k_begin = seg * p.seg_tiles;
  const int k_end = min((L + kTile - 1) / kTile, k_begin + p.seg_tiles);
  const size_t seg_row = row * p.n_seg + seg;

  float a2[kS], Av[kS], h[kS];
#pragma unroll
  for (int j = 0; j < kS; ++j) {
    const int n = st_of(j);
    Av[j] = MSS_SEL(in_bounds(d * NS + n, static_cast<long long>(p.dim) * NS, kSiteA),
                    __ldg(p.A + d * NS + n), 0.f);
    a2[j] = Av[j] * kLog2e;
    float h0 = 0.f;
    if (!kEnd && lane_active) {
      if (seg > 0)
        h0 = MSS_SEL(in_bounds(seg_row * NS + n, n_bd * p.n_seg * NS, kSiteSegIn),
                     p.seg_in[seg_row * NS + n], 0.f);
      else if (p.h0 MSS_AND(in_bounds(row * NS + n, n_bd * NS, kSiteH0)))
        h0 = __ldg(p.h0 + row * NS + n);
    }
    h[j] = h0;
  }
  float dsum = 0.f;  // kEnd: sum of delta_eff over the segment

  const size_t bdl = static_cast<size_t>(b) * p.dim * L;
  const T* u_b = static_cast<const T*>(p.u) + bdl;
  const T* dl_b = static_cast<const T*>(p.delta) + bdl;
  const bool has_z = kStd || p.z != nullptr;
  const bool has_pre = kStd || p.out_pre != nullptr;
  const bool softplus_on = kStd || p.delta_softplus != 0;
  const T* z_b = p.z ? static_cast<const T*>(p.z) + bdl : nullptr;
  T* out_b = static_cast<T*>(p.out) + bdl;
  T* pre_b = p.out_pre ? static_cast<T*>(p.out_pre) + bdl : nullptr;
  const T* B_b = static_cast<const T*>(p.B) + static_cast<size_t>(b) * NS * L;
  const T* C_b = static_cast<const T*>(p.C) + static_cast<size_t>(b) * NS * L;
  const bool use_tma = p.tma_ok != 0;

  // Issues the TMA copies of tile `k` into staging buffer (k - k_begin) % 2
  // (one thread). The end-state pass needs neither z nor C.
  auto issue = [&](int k) {
    const int s = (k - k_begin) & 1;
    const int t0 = k * kTile;
    uint64_t* bar = &sh.bar[s];
    if (t0 >= len) {
      mbar_arrive_expect_tx(bar, 0);
      return;
    }
    constexpr uint32_t kChBytes = kCh * kTile * sizeof(T);
    constexpr uint32_t kNBytes = NS * kTile * sizeof(T);
    const bool with_z = has_z && !kEnd;
    mbar_arrive_expect_tx(bar, (with_z ? 3 : 2) * kChBytes + (kEnd ? 1 : 2) * kNBytes);
    const int rc = b * p.dim + d0;  // first channel row
    tma_load_2d(&sh.rawD[s][0][0], &maps.d, t0, rc, bar);
    tma_load_2d(&sh.rawU[s][0][0], &maps.u, t0, rc, bar);
    if (with_z) tma_load_2d(&sh.rawZ[s][0][0], &maps.z, t0, rc, bar);
    tma_load_2d(&sh.rawB[s][0][0], &maps.b, t0, b * NS, bar);
    if (!kEnd) tma_load_2d(&sh.rawC[s][0][0], &maps.c, t0, b * NS, bar);
  };

  // transform / emit items (4 steps of one channel): lane l of warp w takes
  // steps (l % 8) * 4 .. + 3 of channels w kCPW + l / 8 + k * kItemChStride,
  // i.e. only its own warp's scan channels, so that the work rows pass from
  // transform to scan to emit within the warp
  constexpr int kItems = kCh * (kTile / 4) / kThreads;
  constexpr int kItemChStride = 32 / (kTile / 4);
  static_assert(kItems * kItemChStride == Cfg::kCPW, "a warp's items cover its channels");
  const int it_tt = (lane % (kTile / 4)) * 4;
  const int it_c0 = warp * Cfg::kCPW + lane / (kTile / 4);
  float it_bias[kItems], it_D[kItems];
#pragma unroll
  for (int k = 0; k < kItems; ++k) {
    const int c = it_c0 + k * kItemChStride;
    it_bias[k] = (p.delta_bias && c < n_ch MSS_AND(in_bounds(d0 + c, p.dim, kSiteBias)))
                     ? __ldg(p.delta_bias + d0 + c) : 0.f;
    it_D[k] = (p.D && c < n_ch MSS_AND(in_bounds(d0 + c, p.dim, kSiteD)))
                  ? __ldg(p.D + d0 + c) : 0.f;
  }

  if (use_tma) {
    if (tid == 0) {
      mbar_init(&sh.bar[0], 1);
      mbar_init(&sh.bar[1], 1);
      fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0 && k_begin < k_end) issue(k_begin);
  }

  for (int k = k_begin; k < k_end; ++k) {
    const int kk = k - k_begin;  // position in the segment
    const int s = kk & 1;
    const int t0 = k * kTile;
    if (use_tma) {
      const bool ok = mbar_wait_bounded(&sh.bar[s], (kk >> 1) & 1, p.wait_polls);
      // the CTA's one barrier per tile (TMA staging): past it every warp is
      // done with the previous tile, whose staging buffer the next copies fill
      if (__syncthreads_or(!ok)) {
        // A copy did not complete in time: report it, let the copy in
        // flight into this CTA's staging land (bounded), and leave. Tile k's
        // copies are the only ones in flight: the next tile's are issued
        // only after this wait succeeds.
        if (tid == 0) {
          atomicOr(&g_fwd_device_error, kErrTmaTimeout);
          mbar_wait_bounded(&sh.bar[s], (kk >> 1) & 1);
        }
        return;
      }
      if (tid == 0 && k + 1 < k_end) {
        fence_proxy_async_smem();  // the previous tile's reads of that buffer are done
        issue(k + 1);
      }
    }
    // fp32 B/C read in place from the TMA staging: no CTA-wide widening, and
    // the transform, scan and emit of a channel stay in one warp
    const bool lean = kDirectBC && use_tma;

    // whole tile: every channel live, every step valid, staged by TMA; the
    // transform and emit then run without per-element predicates
    const bool full = use_tma && n_ch == kCh && t0 + kTile <= len;
    if (t0 < len) {
      // ---- 1. transform the tile into fp32 work tiles, 4 steps per item
      auto transform = [&](auto full_t) {
        constexpr bool kFull = decltype(full_t)::value;
#pragma unroll
        for (int k = 0; k < kItems; ++k) {
          const int c = it_c0 + k * kItemChStride, tt = it_tt;
          float x[4] = {0.f, 0.f, 0.f, 0.f}, uv[4] = {0.f, 0.f, 0.f, 0.f};
          if (kFull) {
            load4_smem(&sh.rawD[s][c][tt], x);
            load4_smem(&sh.rawU[s][c][tt], uv);
          } else if (c < n_ch) {
            if (use_tma) {
              load4_smem(&sh.rawD[s][c][tt], x);
              load4_smem(&sh.rawU[s][c][tt], uv);
            } else {
              const size_t off = static_cast<size_t>(d0 + c) * L + t0 + tt;
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                if (t0 + tt + e < len MSS_AND(in_array(dl_b + off + e,
                                                       static_cast<const T*>(p.delta), n_rows,
                                                       kSiteRowIn))) {
                  x[e] = Elem<T>::ld(dl_b + off + e);
                  uv[e] = Elem<T>::ld(u_b + off + e);
                }
              }
            }
          }
          float dv[4], du[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const bool valid = kFull || (c < n_ch && t0 + tt + e < len);
            const float xe = x[e] + it_bias[k];
            const float de = softplus_on ? softplus_f(xe) : xe;
            dv[e] = valid ? de : 0.f;
            du[e] = valid ? (kZOH ? uv[e] : de * uv[e]) : 0.f;
          }
          *reinterpret_cast<float4*>(&sh.dlt[c][tt]) = make_float4(dv[0], dv[1], dv[2], dv[3]);
          *reinterpret_cast<float4*>(&sh.dlu[c][tt]) = make_float4(du[0], du[1], du[2], du[3]);
        }
      };
      if (full) {
        transform(std::true_type{});
      } else {
        transform(std::false_type{});
      }
      if (!(kDirectBC && use_tma)) {
        for (int i = tid; i < NS * (kTile / 4); i += kThreads) {
          const int n = i / (kTile / 4), tt = (i % (kTile / 4)) * 4;
          float bv[4] = {0.f, 0.f, 0.f, 0.f}, cv[4] = {0.f, 0.f, 0.f, 0.f};
          if (use_tma) {
            load4_smem(&sh.rawB[s][n][tt], bv);
            load4_smem(&sh.rawC[s][n][tt], cv);
          } else {
            const size_t off = static_cast<size_t>(n) * L + t0 + tt;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              if (t0 + tt + e < len MSS_AND(in_array(B_b + off + e, static_cast<const T*>(p.B),
                                                     n_bc, kSiteBCIn))) {
                bv[e] = Elem<T>::ld(B_b + off + e);
                cv[e] = Elem<T>::ld(C_b + off + e);
              }
            }
          }
          const float4 b4 = make_float4(bv[0], bv[1], bv[2], bv[3]);
          const float4 c4 = make_float4(cv[0], cv[1], cv[2], cv[3]);
          if constexpr (kDirectBC) {
            // fp32 without TMA: write the layout the TMA swizzle would produce
            const int col = ((tt >> 2) ^ (n & 7)) << 2;
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(&sh.rawB[s][n][0]) + col) = b4;
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(&sh.rawC[s][n][0]) + col) = c4;
          } else {
            *reinterpret_cast<float4*>(&sh.Bs[n][tt]) = b4;
            *reinterpret_cast<float4*>(&sh.Cs[n][tt]) = c4;
          }
        }
      }
      if (lean) {
        __syncwarp();
      } else {
        __syncthreads();  // B/C widened by the whole CTA
      }

      // ---- 2. sequential scan over the tile, 4 steps per iteration; the
      // kLPC lanes of a channel read adjacent B/C rows (distinct banks) and
      // pairs of steps are packed into fp32x2 operations.
      const int steps = min(kTile, len - t0);
      // this lane's B rows as byte offsets into shared memory with the
      // swizzle key folded in: rows are 128-byte aligned, so the 16-byte
      // chunk of group g sits at oB[j] ^ (g << 4)
      const char* const smem_c = reinterpret_cast<const char*>(smem_raw);
      uint32_t oB[kS];
#pragma unroll
      for (int j = 0; j < kS; ++j) {
        const char* row_b = reinterpret_cast<const char*>(&sh.rawB[s][st_of(j)][0]);
        oB[j] = static_cast<uint32_t>(row_b - smem_c) | ((st_of(j) & 7) << 4);
      }
      constexpr int kCfromB = 2 * Sh::kNSP * kTile;  // rawC - rawB, elements
      static_assert(offsetof(Sh, rawC) - offsetof(Sh, rawB) == kCfromB * sizeof(T),
                    "rawC follows rawB");
      const float* const rdl = &sh.dlt[cl][0];
      const float* const rdu = &sh.dlu[cl][0];
      const bool save_carries = kStd || p.chunk_states != nullptr;
      float* cs = p.chunk_states + carry_offset(b, t0 / kCkpt, p.n_chunks, p.dim, d, NS) + q * kS;
      const size_t cs_step = static_cast<size_t>(p.dim) * NS;  // next carry index
      auto scan = [&](auto full_t) {
        constexpr bool kFull = decltype(full_t)::value;
        const int n_steps = kFull ? kTile : steps;
#pragma unroll 4
        for (int tt = 0; tt < n_steps; tt += 4) {
          const float4 dl4 = *reinterpret_cast<const float4*>(rdl + tt);
          const float4 du4 = *reinterpret_cast<const float4*>(rdu + tt);
          const float2 dlp[2] = {make_float2(dl4.x, dl4.y), make_float2(dl4.z, dl4.w)};
          const float2 dup_[2] = {make_float2(du4.x, du4.y), make_float2(du4.z, du4.w)};
          float2 yp2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
          for (int j = 0; j < kS; ++j) {
            const int n = st_of(j);
            float4 B4, C4;
            if constexpr (kDirectBC) {
              // 16-byte chunk tt/4 of row n sits at chunk (tt/4) ^ (n & 7)
              const char* pb = smem_c + (oB[j] ^ static_cast<uint32_t>(tt << 2));
              B4 = *reinterpret_cast<const float4*>(pb);
              C4 = *reinterpret_cast<const float4*>(pb + kCfromB * sizeof(float));
            } else {
              B4 = *reinterpret_cast<const float4*>(&sh.Bs[n][tt]);
              C4 = *reinterpret_cast<const float4*>(&sh.Cs[n][tt]);
            }
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
          if constexpr (kEnd) {
            dsum += (dl4.x + dl4.y) + (dl4.z + dl4.w);
          } else {
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
              sh.dlu[cl][tt + q] = kk;  // step tt + q
            } else if constexpr (kLPC == 2) {
              const bool hi = (q & 1) != 0;
              const float s0 = hi ? yp[0] : yp[2], s1 = hi ? yp[1] : yp[3];
              float k0 = hi ? yp[2] : yp[0], k1 = hi ? yp[3] : yp[1];
              k0 += __shfl_xor_sync(0xffffffffu, s0, 1);
              k1 += __shfl_xor_sync(0xffffffffu, s1, 1);
              sh.dlu[cl][tt + 2 * q] = k0;
              sh.dlu[cl][tt + 2 * q + 1] = k1;
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e) sh.dlu[cl][tt + e] = yp[e];
            }
            // carry after these 4 steps (entries past the valid length are not
            // written: the backward never reads them; none for forward-only calls)
            if (lane_active && save_carries
                    MSS_AND(in_array(cs, p.chunk_states,
                                     n_bd * p.n_chunks * NS - (kS - 1), kSiteCarry))) {
              if constexpr (kS == 4) {
                *reinterpret_cast<float4*>(cs) = make_float4(h[0], h[1], h[2], h[3]);
              } else {
#pragma unroll
                for (int j = 0; j < kS; ++j) cs[j] = h[j];
              }
            }
            cs += cs_step;
          }
        }
      };
      if (full) {
        scan(std::true_type{});
      } else {
        scan(std::false_type{});
      }
    }

    __syncwarp();  // the warp's y rows

    if constexpr (!kEnd) {
      // ---- 3. emit out = (y + D u) * silu(z), and y + D u, 4 steps per item
      auto emit = [&](auto full_t) {
        constexpr bool kFull = decltype(full_t)::value;
#pragma unroll
        for (int k = 0; k < kItems; ++k) {
          const int c = it_c0 + k * kItemChStride, tt = it_tt;
          const int t = t0 + tt;
          if (!kFull && (c >= n_ch || t >= L)) continue;
          const size_t off = static_cast<size_t>(d0 + c) * L + t;
          float o[4] = {0.f, 0.f, 0.f, 0.f}, pre[4] = {0.f, 0.f, 0.f, 0.f};
          if (kFull || t < len) {
            // the raw u and z of this tile are still staged (the buffer is
            // refilled only after the tile's closing barrier)
            float zv[4], uv[4];
            if (kFull || use_tma) {
              load4_smem(&sh.rawU[s][c][tt], uv);
              if (has_z) load4_smem(&sh.rawZ[s][c][tt], zv);
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                uv[e] = t + e < len MSS_AND(in_array(u_b + off + e, static_cast<const T*>(p.u),
                                                     n_rows, kSiteRowIn))
                            ? Elem<T>::ld(u_b + off + e) : 0.f;
                if (has_z)
                  zv[e] = t + e < L MSS_AND(in_array(z_b + off + e, static_cast<const T*>(p.z),
                                                     n_rows, kSiteRowIn))
                              ? Elem<T>::ld(z_b + off + e) : 0.f;
              }
            }
            const float4 y4 = *reinterpret_cast<const float4*>(&sh.dlu[c][tt]);
            const float ys4[4] = {y4.x, y4.y, y4.z, y4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              if (kFull || t + e < len) {
                pre[e] = fmaf(it_D[k], uv[e], ys4[e]);
                o[e] = has_z ? pre[e] * silu_f(zv[e]) : pre[e];
              }
            }
          }
          MSS_BOUNDS_ONLY(
              if (!in_array(out_b + off, static_cast<T*>(p.out), n_rows, kSiteOut) ||
                  !in_array(out_b + off + min(4, L - t) - 1, static_cast<T*>(p.out), n_rows,
                            kSiteOut)) continue;)
          if (kFull || use_tma) {  // whole, aligned groups: L is a multiple of 4 here
            store4_global(out_b + off, o);
            if (has_pre) store4_global(pre_b + off, pre);
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              if (t + e < L) {
                Elem<T>::st(out_b + off + e, o[e]);
                if (has_pre) Elem<T>::st(pre_b + off + e, pre[e]);
              }
            }
          }
        }
      };
      if (full) {
        emit(std::true_type{});
      } else {
        emit(std::false_type{});
      }
    }
    // with TMA the next tile's barrier follows its wait; plain staging keeps
    // the widened B/C of this tile until every warp has scanned it
    if (!use_tma) __syncthreads();
  }

  if constexpr (kEnd) {
    if (lane_active) {
#pragma unroll
      for (int j = 0; j < kS; ++j)
        MSS_IF(in_bounds(seg_row * NS + st_of(j), n_bd * p.n_seg * NS, kSiteSegEnd))
        p.seg_end[seg_row * NS + st_of(j)] = h[j];
      if (q == 0 MSS_AND(in_bounds(seg_row, n_bd * p.n_seg, kSiteSegDsum)))
        p.seg_dsum[seg_row] = dsum;
    }
  } else if (p.last_state && lane_active && seg == p.n_seg - 1) {
#pragma unroll
    for (int j = 0; j < kS; ++j)
      MSS_IF(in_bounds(row * NS + st_of(j), n_bd * NS, kSiteLast))
      p.last_state[row * NS + st_of(j)] = h[j];
  }
}

// Entering state of every time segment, in order: segment 0 starts from h0
// (or zero), segment s + 1 from a_seg(s) * in(s) + end(s), where end(s) is
// segment s's end state from a zero start and a_seg(s) = 2^(A log2 e *
// sum of delta_eff over s) its decay. One thread per (batch, channel, state).
__global__ void seg_combine_fwd_kernel(const float* __restrict__ A, const float* __restrict__ h0,
                                       float* seg_end, float* seg_dsum, float* seg_in,
                                       int batch, int dim, int dstate, int n_seg) {
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i >= static_cast<long long>(batch) * dim * dstate) return;
  const int n = static_cast<int>(i % dstate);
  const long long bd = i / dstate;
  const int d = static_cast<int>(bd % dim);
  const float a2 = A[static_cast<size_t>(d) * dstate + n] * kLog2e;
  float h = h0 ? h0[i] : 0.f;
  for (int s = 0; s < n_seg; ++s) {
    const size_t sr = static_cast<size_t>(bd) * n_seg + s;
    seg_in[sr * dstate + n] = h;
    if (s + 1 < n_seg) {
      h = fmaf(exp2f(a2 * seg_dsum[sr]), h, seg_end[sr * dstate + n]);
    } else {
      // the last segment has no end-state pass: keep its slots defined
      seg_end[sr * dstate + n] = 0.f;
      if (n == 0) seg_dsum[sr] = 0.f;
    }
  }
}

// Whether the grid rows take the batches longest first (right padding, one
// time segment).
static bool longest_first(const FwdParams& p) {
  return p.seq_lens != nullptr && p.n_seg == 1 && p.batch <= kLongestFirstMax;
}

template <int NS, typename T, bool kZOH>
static cudaError_t launch_fwd_t(const FwdParams& p, const FwdMaps& maps, bool wide,
                                cudaStream_t stream) {
  if constexpr (NS == 16) {
    if (wide) {  // unsegmented only
      using CfgW = FwdCfg<NS, true>;
      const size_t smem_w = sizeof(FwdShared<NS, T, true>);
      const bool std_call = p.delta_softplus != 0 && p.z != nullptr && p.out_pre != nullptr &&
                            p.chunk_states != nullptr;
      auto kern_w = longest_first(p)
                        ? (std_call ? ss_fwd_kernel<NS, T, kZOH, false, true, true, true>
                                    : ss_fwd_kernel<NS, T, kZOH, false, true, true>)
                        : (std_call ? ss_fwd_kernel<NS, T, kZOH, false, true, false, true>
                                    : ss_fwd_kernel<NS, T, kZOH, false, true>);
      cudaError_t e = cudaFuncSetAttribute(
          kern_w, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem_w));
      if (e != cudaSuccess) return e;
      const unsigned gxw = (p.dim + CfgW::kCh - 1) / CfgW::kCh;
      kern_w<<<dim3(gxw, p.batch, 1), CfgW::kThreads, smem_w, stream>>>(p, maps);
      return cudaPeekAtLastError();
    }
  }
  using Cfg = FwdCfg<NS>;
  const size_t smem = sizeof(FwdShared<NS, T>);
  auto kern = ss_fwd_kernel<NS, T, kZOH, false, false>;
  if constexpr (NS == 16) {
    const bool std_call = p.delta_softplus != 0 && p.z != nullptr && p.out_pre != nullptr &&
                          p.chunk_states != nullptr;
    if (longest_first(p)) {
      kern = ss_fwd_kernel<NS, T, kZOH, false, false, true>;
    } else if (std_call) {
      kern = ss_fwd_kernel<NS, T, kZOH, false, false, false, true>;
    }
  }
  auto kern_end = ss_fwd_kernel<NS, T, kZOH, true, false>;
  cudaError_t e = cudaFuncSetAttribute(
      kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const unsigned gx = (p.dim + Cfg::kCh - 1) / Cfg::kCh;
  if (p.n_seg > 1) {
    e = cudaFuncSetAttribute(kern_end, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    kern_end<<<dim3(gx, p.batch, p.n_seg - 1), Cfg::kThreads, smem, stream>>>(p, maps);
    const long long total = static_cast<long long>(p.batch) * p.dim * NS;
    seg_combine_fwd_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
        p.A, p.h0, p.seg_end, p.seg_dsum, const_cast<float*>(p.seg_in), p.batch, p.dim, NS,
        p.n_seg);
  }
  kern<<<dim3(gx, p.batch, p.n_seg), Cfg::kThreads, smem, stream>>>(p, maps);
  return cudaPeekAtLastError();
}

template <typename T, bool kZOH>
static cudaError_t launch_fwd_n(const FwdParams& p, const FwdMaps& maps, int dstate, bool wide,
                                cudaStream_t stream) {
  switch (dstate) {
    case 1: return launch_fwd_t<1, T, kZOH>(p, maps, false, stream);
    case 2: return launch_fwd_t<2, T, kZOH>(p, maps, false, stream);
    case 4: return launch_fwd_t<4, T, kZOH>(p, maps, false, stream);
    case 8: return launch_fwd_t<8, T, kZOH>(p, maps, false, stream);
    case 16: return launch_fwd_t<16, T, kZOH>(p, maps, wide, stream);
    default: return cudaErrorInvalidValue;
  }
}

static int fwd_channels_per_cta(int dstate) {
  switch (dstate) {
    case 1: return FwdCfg<1>::kCh;
    case 2: return FwdCfg<2>::kCh;
    case 4: return FwdCfg<4>::kCh;
    case 8: return FwdCfg<8>::kCh;
    default: return FwdCfg<16>::kCh;
  }
}
static_assert(FwdCfg<16>::kCh == 8 && FwdCfg<8>::kCh == 16 && FwdCfg<4>::kCh == 32 &&
                  FwdCfg<2>::kCh == 32 && FwdCfg<1>::kCh == 32 && kTile == kScanTile,
              "seg_plan's CTA count");

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  return fn;
}

// Row-major [rows][L] tensor, boxes of [box_rows][kTile]; zero fill outside.
static bool encode_rows(CUtensorMap* m, const void* base, int io_dtype, uint64_t rows,
                        uint64_t L, uint32_t box_rows, bool swizzle128 = false) {
  auto fn = tensor_map_encoder();
  if (!fn) return false;
  const size_t esize = io_dtype == MSS_BF16 ? 2 : 4;
  const cuuint64_t dims[2] = {L, rows};
  const cuuint64_t strides[1] = {L * esize};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kTile), box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, io_dtype == MSS_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
            2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool aligned16(const void* ptr) {
  return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0;
}

cudaError_t launch_fwd(const FwdParams& p_in, int dstate, int io_dtype, int zoh,
                       cudaStream_t stream) {
  FwdParams p = p_in;
  const size_t esize = io_dtype == MSS_BF16 ? 2 : 4;
  // time segments; their scratch follows the carries in chunk_states
  // (a forward-only call without chunk_states runs unsegmented: the segment
  // scratch lives in chunk_states)
  const SegPlan sp = p.chunk_states ? seg_plan(p.batch, p.seqlen, p.dim, dstate)
                                    : SegPlan{1, (p.seqlen + kTile - 1) / kTile};
  p.n_seg = sp.n_seg;
  p.seg_tiles = sp.seg_tiles;
  if (p.n_seg > 1) {
    const size_t bds = static_cast<size_t>(p.batch) * p.dim * p.n_seg;
    float* scratch = p.chunk_states + static_cast<size_t>(p.batch) * p.n_chunks * p.dim * dstate;
    p.seg_end = scratch;
    p.seg_in = scratch + bds * dstate;
    p.seg_dsum = scratch + 2 * bds * dstate;
  }
  // four-warp CTAs (N = 16) once the one-warp grid fills the GPU (8 or more
  // CTAs per SM); smaller grids keep the finer one-warp work units
  const long long narrow_ctas =
      static_cast<long long>(p.batch) * ((p.dim + FwdCfg<16>::kCh - 1) / FwdCfg<16>::kCh);
  bool wide = narrow_ctas >= 148LL * 8;
  if (const char* env = getenv("MAMBA_SS_FWD_WIDE")) wide = atoi(env) != 0;  // tests force it
  wide = wide && dstate == 16 && p.n_seg == 1;
  // TMA needs 16-byte aligned bases and row strides (L * esize).
  p.tma_ok = (p.seqlen * esize) % 16 == 0 && aligned16(p.u) && aligned16(p.delta) &&
             aligned16(p.B) && aligned16(p.C) && (!p.z || aligned16(p.z));
  FwdMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (p.tma_ok) {
    const uint64_t rows = static_cast<uint64_t>(p.batch) * p.dim;
    const uint64_t brows = static_cast<uint64_t>(p.batch) * dstate;
    const uint32_t ch = static_cast<uint32_t>(wide ? FwdCfg<16, true>::kCh
                                                    : fwd_channels_per_cta(dstate));
    const uint64_t L = p.seqlen;
    p.tma_ok = encode_rows(&maps.d, p.delta, io_dtype, rows, L, ch) &&
               encode_rows(&maps.u, p.u, io_dtype, rows, L, ch) &&
               (!p.z || encode_rows(&maps.z, p.z, io_dtype, rows, L, ch)) &&
               encode_rows(&maps.b, p.B, io_dtype, brows, L, dstate, io_dtype == MSS_F32) &&
               encode_rows(&maps.c, p.C, io_dtype, brows, L, dstate, io_dtype == MSS_F32);
  }
  if (io_dtype == MSS_BF16) {
    return zoh ? launch_fwd_n<__nv_bfloat16, true>(p, maps, dstate, wide, stream)
               : launch_fwd_n<__nv_bfloat16, false>(p, maps, dstate, wide, stream);
  }
  return zoh ? launch_fwd_n<float, true>(p, maps, dstate, wide, stream)
             : launch_fwd_n<float, false>(p, maps, dstate, wide, stream);
}

unsigned int take_fwd_device_error() {
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_fwd_device_error, sizeof(v)) != cudaSuccess) return ~0u;
  cudaMemcpyToSymbol(g_fwd_device_error, &zero, sizeof(zero));
  return v;
}

void take_fwd_bounds(unsigned long long out[4]) { take_oob_record(out); }

// One thread checks index n + 7 against extent n without touching memory:
// the bounds build must count and record it (site kSiteSelfTest).
__global__ void bounds_selftest_kernel(long long n) {
  if (threadIdx.x == 0 && blockIdx.x == 0) (void)in_bounds(n + 7, n, kSiteSelfTest);
}

cudaError_t launch_bounds_selftest(long long n) {
  bounds_selftest_kernel<<<1, 32>>>(n);
  return cudaPeekAtLastError();
}

}  // namespace mss

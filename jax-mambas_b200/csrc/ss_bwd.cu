// Backward selective scan for sm_100a.
//
// Replaces selective_scan_bwd_kernel (native/upstream_mamba/
// selective_scan_bwd_kernel.cuh:65-497) and SelectiveScanBackwardImpl
// (native/selective_scan_bwd.cu:24-162), and adds the gradients of the fused
// softplus(delta + bias), D skip and silu(z) gate, and the ZOH discretization
// the reference leaves to JAX autodiff (mamba/selective_scan_cuda.py:250-256).
//
// The scan kernel (ss_bwd_tile_kernel) is described below; after it,
// reduce_params_kernel sums the per-batch dA, dD and ddelta_bias partials in a
// fixed order and, for bf16 I/O, f32_to_bf16_kernel narrows dB and dC.
#include <algorithm>
#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <type_traits>

#include "ss_common.cuh"
#include "ss_launch.h"

namespace mss {

__device__ unsigned int g_bwd_device_error = 0;

// ============================================================================
// Tile backward: sequential in time inside each lane.
//
// A lane owns kS states of one channel, kLPC = NS / kS lanes a channel, and a
// one-warp CTA kCh = 32 / kLPC channels of one batch (the forward's
// decomposition). The forward saves the state after every kGrp = 4 steps,
// so groups are independent given their entering state. The CTA walks
// kBT-step tiles in reverse; per tile
//   0. TMA stages delta, u, dout, z, pre-gate ([kCh channels x kBT steps])
//      and B, C ([N x kBT]) with the 128-byte (fp32) / 64-byte (bf16)
//      swizzle; the next tile's copies fly while this one computes;
//   1. transform: delta_eff = softplus(delta + bias) and dy = dout silu(z)
//      become fp32 work rows (for fp32 I/O in place of delta and dout), and
//      dz = dout pre silu'(z) is written in place of z;
//   2. the saved state entering each group is loaded into registers;
//   3. groups in reverse: recompute a_t, h_t over the group, run the adjoint
//      g_t = dy_t C_t + a_{t+1} g_{t+1} per state, and form per step
//      sum_n g B and sum_n g A a h_{t-1} (summed over the channel's lanes,
//      then du, ddelta written in place of u and delta), per lane dA, and
//      dB = g delta u, dC = dy h per (channel, state) into a shared tile that
//      the warp sums over channels and adds to the fp32 accumulators with
//      16-byte atomics;
//   4. the tile's du, ddelta and dz leave by TMA bulk stores.
// Shared memory is kept under 20 KB per CTA (fp32, N = 16) so that a
// Mamba-130M layer's CTAs are all resident at once (11 per SM).
// ============================================================================
constexpr int kBT = 32;         // steps per tile
constexpr int kGrp = kCkpt;     // steps per group (one saved carry per group)
constexpr int kNG = kBT / kGrp;  // groups per tile

template <int NS>
struct TileCfg {
  static constexpr int kS = NS < 4 ? NS : 4;  // states per lane
  static constexpr int kLPC = NS / kS;        // lanes per channel
  static constexpr int kCh = 32 / kLPC;       // channels per CTA (one warp)
  // column swizzle of the [channel][state] dB/dC tile: the 32 lanes' float4
  // writes of one state index, and the flush's row reads, avoid bank conflicts
  static __device__ __forceinline__ int part_swz(int c) { return mss::part_swz<NS>(c); }
};

struct TileMaps {
  CUtensorMap d, u, y, z, p, b, c;  // loads: [rows][L], boxes [box rows][kBT]
  CUtensorMap du, dd, dz;           // stores
};

// kW warps per CTA (N = 16 only: 2): the warps share the staging of B and
// C and every TMA copy covers all kCh channels of the CTA; with more than one
// warp the pre-gate rows are double-buffered with the other arrays, so that
// the CTA needs one barrier per tile.
template <int NS, typename T, int kW = 1>
struct TileShared {
  static constexpr int kCh = TileCfg<NS>::kCh * kW;
  static constexpr int kNSP = NS < 8 ? 8 : NS;  // whole swizzle atoms
  static constexpr int kPB = kW > 1 ? 2 : 1;    // pre-gate buffers
  static constexpr bool kInPlace = sizeof(T) == 4;  // fp32 work rows live in rawD / rawY
  alignas(1024) T rawD[2][kCh][kBT];  // delta in; (fp32: delta_eff;) ddelta out
  alignas(1024) T rawU[2][kCh][kBT];  // u in, du out
  alignas(1024) T rawY[2][kCh][kBT];  // dout in; (fp32: dy)
  alignas(1024) T rawZ[2][kCh][kBT];  // z in, dz out
  // B and C staged as fp32 whatever the I/O type (bf16 I/O: from the
  // launcher's widened copies), read in place through the 128-byte swizzle
  alignas(1024) float rawB[2][kNSP][kBT];
  alignas(1024) float rawC[2][kNSP][kBT];
  alignas(1024) T rawP[kPB][kCh][kBT];  // pre-gate output (read by the transform only)
  // bf16 I/O: fp32 work rows delta_eff and dy, swizzled like fp32 staging
  alignas(16) float wD[kInPlace ? 1 : kCh][kBT];
  alignas(16) float wY[kInPlace ? 1 : kCh][kBT];
  // one group's dB or dC per (channel, swizzled state); N = 16 sums by shuffles
  float4 part[NS == 16 ? 1 : kCh][NS];
  uint64_t bar[2];
  uint64_t barP;
};

// Element (r, t) of a staged [rows][kBT] tile: fp32 rows are 128 bytes under
// the 128-byte swizzle (16-byte chunk j of row r at j ^ (r & 7)), bf16 rows
// 64 bytes under the 64-byte swizzle (chunk j at j ^ ((r >> 1) & 3)).
__device__ __forceinline__ int sw_idx(const float*, int r, int t) {
  return r * kBT + ((((t >> 2) ^ (r & 7)) << 2) | (t & 3));
}
__device__ __forceinline__ int sw_idx(const __nv_bfloat16*, int r, int t) {
  return r * kBT + ((((t >> 3) ^ ((r >> 1) & 3)) << 3) | (t & 7));
}

// The same addressing split into a per-row part (row pointer, swizzle key,
// computed once per tile) and a per-group part: group g's steps 4g .. 4g+3
// of a row start grp_off(row key, g) elements after the row pointer.
__device__ __forceinline__ int row_key(const float*, int r) { return r & 7; }
__device__ __forceinline__ int row_key(const __nv_bfloat16*, int r) { return (r >> 1) & 3; }
__device__ __forceinline__ int grp_off(const float*, int key, int g) { return (g ^ key) << 2; }
__device__ __forceinline__ int grp_off(const __nv_bfloat16*, int key, int g) {
  return (((g >> 1) ^ key) << 3) | ((g & 1) << 2);
}
__device__ __forceinline__ float4 ld4p(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}
__device__ __forceinline__ float4 ld4p(const __nv_bfloat16* p) {
  return bf16x4_to_f32(*reinterpret_cast<const uint2*>(p));
}

// Steps t .. t+3 (t a multiple of 4) of row r as fp32.
__device__ __forceinline__ float4 ld4s(const float* tile, int r, int t) {
  return *reinterpret_cast<const float4*>(tile + sw_idx(tile, r, t));
}
__device__ __forceinline__ float4 ld4s(const __nv_bfloat16* tile, int r, int t) {
  return bf16x4_to_f32(*reinterpret_cast<const uint2*>(tile + sw_idx(tile, r, t)));
}
__device__ __forceinline__ void st4s(float* tile, int r, int t, float4 v) {
  *reinterpret_cast<float4*>(tile + sw_idx(tile, r, t)) = v;
}
__device__ __forceinline__ void st4s(__nv_bfloat16* tile, int r, int t, float4 v) {
  uint2 w;
  *reinterpret_cast<__nv_bfloat162*>(&w.x) = __floats2bfloat162_rn(v.x, v.y);
  *reinterpret_cast<__nv_bfloat162*>(&w.y) = __floats2bfloat162_rn(v.z, v.w);
  *reinterpret_cast<uint2*>(tile + sw_idx(tile, r, t)) = w;
}
template <typename T>
__device__ __forceinline__ float ld1s(const T* tile, int r, int t) {
  return to_f32(tile[sw_idx(tile, r, t)]);
}
template <typename T>
__device__ __forceinline__ void st1s(T* tile, int r, int t, float v) {
  tile[sw_idx(tile, r, t)] = static_cast<T>(v);
}

// Plain-load staging of a [box_rows][kBT] tile in the TMA's swizzled layout:
// rows at or past n_valid and steps at or past L read as zero (one warp).
template <typename T>
__device__ void stage_tile_plain(T* tile, const T* base, size_t row0, int n_valid, int box_rows,
                                 int L, int t0, int lane, long long extent) {
  (void)extent;  // element count of base (bounds build)
  for (int i = lane; i < box_rows * kBT; i += 32) {
    const int r = i / kBT, t = i % kBT;
    T v = static_cast<T>(0.f);
    if (r < n_valid && t0 + t < L
        MSS_AND(in_bounds(static_cast<long long>((row0 + r) * static_cast<size_t>(L) + t0 + t),
                          extent, kSiteRowIn)))
      v = base[(row0 + r) * static_cast<size_t>(L) + t0 + t];
    tile[sw_idx(tile, r, t)] = v;
  }
}

// Plain stores of a staged tile's rows below n_valid, steps below L (one warp).
template <typename T>
__device__ void unstage_tile_plain(T* base, const T* tile, size_t row0, int n_valid, int L,
                                   int t0, int lane, long long extent) {
  (void)extent;  // element count of base (bounds build)
  for (int i = lane; i < n_valid * kBT; i += 32) {
    const int r = i / kBT, t = i % kBT;
    if (t0 + t < L
        MSS_AND(in_bounds(static_cast<long long>((row0 + r) * static_cast<size_t>(L) + t0 + t),
                          extent, kSiteRowOut)))
      base[(row0 + r) * static_cast<size_t>(L) + t0 + t] = tile[sw_idx(tile, r, t)];
  }
}

// Zeroes steps [from, to) of n rows of length L (one warp); 16-byte stores
// when `vec` (from and to multiples of 16 bytes).
template <typename T>
__device__ void zero_rows(T* base, size_t row0, int n, int L, int from, int to, bool vec,
                          int lane, long long extent) {
  (void)extent;  // element count of base (bounds build)
  if (from >= to) return;
  constexpr int kPer = 16 / sizeof(T);
  for (int r = 0; r < n; ++r) {
    T* rowp = base + (row0 + r) * static_cast<size_t>(L);
    if (vec) {
      for (int t = from + lane * kPer; t < to; t += 32 * kPer)
        MSS_IF(in_array(rowp + t, base, extent, kSiteRowOut) &&
               in_array(rowp + t + kPer - 1, base, extent, kSiteRowOut))
        *reinterpret_cast<uint4*>(rowp + t) = make_uint4(0u, 0u, 0u, 0u);
    } else {
      for (int t = from + lane; t < to; t += 32)
        MSS_IF(in_array(rowp + t, base, extent, kSiteRowOut))
        rowp[t] = static_cast<T>(0.f);
    }
  }
}


// kSeg: the launch is cut into time segments (blockIdx.z); without it the
// segment bounds are compile-time constants (one segment of the whole row).
// kLPT: right-padded batches, grid rows take the sequences longest first
// (batch_of_row); its bound of 16 CTAs per SM keeps the registers at the plain
// kernel's 128 (the ranking code otherwise lifts them to ~170, which cuts the
// resident warps per SM from 16 to 12). 0 leaves the bound to the compiler.
// Two-warp CTAs are bounded to 7 per SM: at 8 (128 registers) the compiler
// spilled 20 bytes and configs[2]'s backward took 3.60 ms, at 7 it does not
// spill (3.55 ms); the group loop unrolled by 1 or 4 measured 3.59 / 3.96 ms.
// kWarps: warps per CTA (TileShared); the CTA's kCh channels are kWarps
// blocks of kCPW, one per warp.
// kStd: the fused layer's usual call (softplus on delta, a z gate, dB/dC by
// atomics), with those three choices compiled in instead of tested per group.
template <int NS, typename T, bool kZOH, bool kSeg, bool kLPT = false, int kWarps = 1,
          bool kStd = false>
__global__ void __launch_bounds__(32 * kWarps, kLPT ? (kWarps == 1 ? 16 : 7) : 0)
    ss_bwd_tile_kernel(const BwdParams p, const __grid_constant__ TileMaps maps) {
  using Cfg = TileCfg<NS>;
  using Sh = TileShared<NS, T, kWarps>;
  constexpr int kS = Cfg::kS;
  constexpr int kLPC = Cfg::kLPC;
  constexpr int kCPW = Cfg::kCh;  // channels per warp
  constexpr int kCh = Sh::kCh;    // channels per CTA
  static_assert(kWarps == 1 || NS == 16, "multi-warp CTAs are for N = 16");
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  Sh& sh = *reinterpret_cast<Sh*>(smem_raw);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int b = kLPT ? batch_of_row(p.seq_lens, p.batch, p.seqlen, static_cast<int>(blockIdx.y))
                     : static_cast<int>(blockIdx.y);
  const int d0 = blockIdx.x * kCh;
  const int L = p.seqlen;
  const int n_ch = min(kCh, p.dim - d0);
  const int c = warp * kCPW + lane / kLPC;  // channel slot in the CTA
  const int q = lane % kLPC;  // lane q owns states q, q + kLPC, ...
  // this warp's block of channel rows: [wc0, wc0 + n_wch)
  const int wc0 = warp * kCPW;
  const int n_wch = max(0, min(kCPW, n_ch - wc0));
  const bool act = c < n_ch;
  const int d = d0 + (act ? c : 0);
  const size_t row = static_cast<size_t>(b) * p.dim + d;
  const size_t row0 = static_cast<size_t>(b) * p.dim + d0;  // first row of the CTA
  // N = 16: dB/dC are summed over the warp's 8 channels by a shuffle
  // reduce-scatter. Lane slot j holds state q + 4 (j ^ perm), perm taken from
  // channel bits 1 and 2, so that the first two shuffle levels exchange the
  // same slots on every lane.
  constexpr bool kShflFlush = NS == 16;
  const int perm = state_perm<NS>(c);
  auto st_of = [&](int j) { return q + kLPC * (j ^ perm); };

  int len = L;
  if (p.seq_lens MSS_AND(in_bounds(b, p.batch, kSiteSeqLens)))
    len = max(0, min(L, p.seq_lens[b]));
  // extents of the arrays, in elements (the staging helpers check against
  // them in the bounds build only)
  const long long n_bd = static_cast<long long>(p.batch) * p.dim;
  const long long n_rows = n_bd * L, n_bc = static_cast<long long>(p.batch) * NS * L;
  // this CTA's time segment: tiles [k_begin, k_end); k_last is the last tile
  // of it with valid steps (k_last < k_begin: none)
  const int seg = kSeg ? static_cast<int>(blockIdx.z) : 0;
  const int n_seg = kSeg ? p.n_seg : 1;
  const int k_begin = kSeg ? seg * p.seg_tiles : 0;
  const int k_end = kSeg ? min((L + kBT - 1) / kBT, k_begin + p.seg_tiles) : (L + kBT - 1) / kBT;
  const int k_last = len > 0 ? min((len - 1) / kBT, k_end - 1) : k_begin - 1;
  const size_t seg_row = row * n_seg + seg;
  const bool use_tma = p.tma_ok != 0;
  const bool tma_store = use_tma && n_ch == kCh;  // whole boxes stay in this batch
  const bool has_z = kStd || p.z != nullptr;
  const bool softplus_on = kStd || p.delta_softplus != 0;

  float Av[kS], a2[kS];
#pragma unroll
  for (int j = 0; j < kS; ++j) {
    Av[j] = MSS_SEL(in_bounds(d * NS + st_of(j), static_cast<long long>(p.dim) * NS, kSiteA),
                    __ldg(p.A + d * NS + st_of(j)), 0.f);
    a2[j] = Av[j] * kLog2e;
  }
  const float Dv = p.D MSS_AND(in_bounds(d, p.dim, kSiteD)) ? __ldg(p.D + d) : 0.f;
  const float bias =
      p.delta_bias MSS_AND(in_bounds(d, p.dim, kSiteBias)) ? __ldg(p.delta_bias + d) : 0.f;

  // Steps past the last valid tile are padding: their gradients are zero.
  {
    const int tz = max(k_last + 1, k_begin) * kBT;
    const int te = min(k_end * kBT, L);
    const bool vec = use_tma;  // 16-byte aligned rows (L * esize % 16 == 0)
    zero_rows(static_cast<T*>(p.du), row0 + wc0, n_wch, L, tz, te, vec, lane, n_rows);
    zero_rows(static_cast<T*>(p.ddelta), row0 + wc0, n_wch, L, tz, te, vec, lane, n_rows);
    if (has_z) zero_rows(static_cast<T*>(p.dz), row0 + wc0, n_wch, L, tz, te, vec, lane, n_rows);
  }

  // TMA pipeline: position i of the walk is tile k_last - i; its arrays go
  // to buffer i & 1 (bar[i & 1]). One warp: its pre-gate rows go to the
  // single rawP (barP, issued once the previous position's transform has
  // read rawP). Several warps: the pre-gate rows travel with the other
  // arrays in buffer i & 1, and the CTA meets one barrier per tile, after the
  // transform: past it every warp is done with position i - 1, whose rows
  // thread 0 then stores and whose buffer it refills with position i + 1.
  constexpr uint32_t kChBytes = kCh * kBT * sizeof(T);
  constexpr uint32_t kNBytes = NS * kBT * sizeof(float);
  const int rc = static_cast<int>(row0);
  auto issue = [&](int i) {  // one thread
    const int s = i & 1;
    const int x = (k_last - i) * kBT;
    uint64_t* bar = &sh.bar[s];
    const uint32_t n_ch_arrays = (has_z ? 4u : 3u) + (kWarps > 1 && has_z ? 1u : 0u);
    mbar_arrive_expect_tx(bar, n_ch_arrays * kChBytes + 2u * kNBytes);
    tma_load_2d(&sh.rawD[s][0][0], &maps.d, x, rc, bar);
    tma_load_2d(&sh.rawU[s][0][0], &maps.u, x, rc, bar);
    tma_load_2d(&sh.rawY[s][0][0], &maps.y, x, rc, bar);
    if (has_z) tma_load_2d(&sh.rawZ[s][0][0], &maps.z, x, rc, bar);
    if (kWarps > 1 && has_z) tma_load_2d(&sh.rawP[s % Sh::kPB][0][0], &maps.p, x, rc, bar);
    tma_load_2d(&sh.rawB[s][0][0], &maps.b, x, b * NS, bar);
    tma_load_2d(&sh.rawC[s][0][0], &maps.c, x, b * NS, bar);
  };
  auto issue_pre = [&](int i) {  // one thread (one-warp CTAs)
    mbar_arrive_expect_tx(&sh.barP, kChBytes);
    tma_load_2d(&sh.rawP[0][0], &maps.p, (k_last - i) * kBT, rc, &sh.barP);
  };
  // the du / ddelta / dz rows of position i (multi-warp CTAs, thread 0)
  auto store_pos = [&](int i) {
    const int s = i & 1;
    const int x = (k_last - i) * kBT;
    MSS_BOUNDS_ONLY(if (!in_bounds(x, L, kSiteTmaStore) ||
                        !in_bounds(rc + kCh - 1, n_bd, kSiteTmaStore)) return;)
    tma_store_2d(&maps.du, x, rc, &sh.rawU[s][0][0]);
    tma_store_2d(&maps.dd, x, rc, &sh.rawD[s][0][0]);
    if (has_z) tma_store_2d(&maps.dz, x, rc, &sh.rawZ[s][0][0]);
    bulk_commit();
  };
  if (use_tma && tid == 0) {
    mbar_init(&sh.bar[0], 1);
    mbar_init(&sh.bar[1], 1);
    mbar_init(&sh.barP, 1);
    fence_mbar_init();
    if (k_last >= k_begin) {
      issue(0);
      if (kWarps == 1 && has_z) issue_pre(0);
    }
    if (k_last >= k_begin + 1) issue(1);
  }
  if constexpr (kWarps > 1) {
    __syncthreads();
  } else {
    __syncwarp();
  }

  // Adjoint carries: g of the step after the current one and its a.
  float gn[kS], an[kS];
  float2 dAacc[kS];
#pragma unroll
  for (int j = 0; j < kS; ++j) {
    // the last segment starts from dlast, the others from the carry their
    // right neighbours pass
    if (kSeg && seg < n_seg - 1)
      gn[j] = act MSS_AND(in_bounds(seg_row * NS + st_of(j), n_bd * n_seg * NS, kSiteSegCarry))
                  ? p.seg_carry[seg_row * NS + st_of(j)] : 0.f;
    else
      gn[j] = (act && p.dlast MSS_AND(in_bounds(row * NS + st_of(j), n_bd * NS, kSiteDlast)))
                  ? __ldg(p.dlast + row * NS + st_of(j)) : 0.f;
    an[j] = 1.f;
    dAacc[j] = make_float2(0.f, 0.f);
  }
  float dD_acc = 0.f, dbias_acc = 0.f;
  const bool acc_aligned = (L & 3) == 0 && ((reinterpret_cast<uintptr_t>(p.dB_acc) |
                                              reinterpret_cast<uintptr_t>(p.dC_acc)) & 15) == 0;
  // deterministic mode: this warp's column of the partial sums instead of
  // the accumulators, written instead of added
  const bool det = !kStd && p.dBC_part != nullptr;
  const int col = static_cast<int>(blockIdx.x) * kWarps + warp;
  float* const part_b =
      det ? p.dBC_part + static_cast<size_t>(b * p.n_cols + col) * 2 * NS * L : nullptr;
  float* dB_b = det ? part_b : p.dB_acc + static_cast<size_t>(b) * NS * L;
  float* dC_b = det ? part_b + static_cast<size_t>(NS) * L : p.dC_acc + static_cast<size_t>(b) * NS * L;

  for (int k = k_last; k >= k_begin; --k) {
    const int i = k_last - k;
    const int s = i & 1;
    const int t0 = k * kBT;
    T* bD = &sh.rawD[s][0][0];
    T* bU = &sh.rawU[s][0][0];
    T* bY = &sh.rawY[s][0][0];
    T* bZ = &sh.rawZ[s][0][0];
    T* bP = &sh.rawP[kWarps > 1 ? s : 0][0][0];
    const float* bB = &sh.rawB[s][0][0];
    const float* bC = &sh.rawC[s][0][0];
    // fp32 work rows: delta_eff and dy
    float* wD = Sh::kInPlace ? reinterpret_cast<float*>(bD) : &sh.wD[0][0];
    float* wY = Sh::kInPlace ? reinterpret_cast<float*>(bY) : &sh.wY[0][0];

    // ---- 2. the saved state entering each group, in slot order (lane q,
    // slot j: state st_of(j), as the forward keeps it); groups starting at or
    // past the valid length carry delta = 0 and only need a finite state.
    // The walk below prefetches two groups ahead so that the loads' latency
    // hides behind the work of the groups in between.
    // carry entering group g sits at carry index t0 / kCkpt + g - 1; the
    // pointer below is that of group kNG - 1 and steps back one index per group
    const size_t cs_step = static_cast<size_t>(p.dim) * NS;
    const float* cs_g = p.chunk_states + q * kS +
                        carry_offset(b, max(t0 / kCkpt + kNG - 2, 0), p.n_chunks, p.dim, d, NS);
    auto load_carry = [&](int g, const float* cs) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      const int gi = t0 / kCkpt + g;  // carry index of the group
      if (act && t0 + g * kGrp < len) {
        if (gi > 0) {
          MSS_IF(in_array(cs, p.chunk_states, n_bd * p.n_chunks * NS, kSiteCarry) &&
                 in_array(cs + kS - 1, p.chunk_states, n_bd * p.n_chunks * NS, kSiteCarry))
          {
            if constexpr (kS == 4) {
              v = *reinterpret_cast<const float4*>(cs);
            } else {
              v.x = cs[0];
              if constexpr (kS > 1) v.y = cs[1];
            }
          }
        } else if (p.h0 MSS_AND(in_bounds(row * NS + NS - 1, n_bd * NS, kSiteH0))) {
          const float* h0 = p.h0 + row * NS;
          v.x = __ldg(h0 + st_of(0));
          if constexpr (kS > 1) v.y = __ldg(h0 + st_of(1));
          if constexpr (kS > 2) {
            v.z = __ldg(h0 + st_of(2));
            v.w = __ldg(h0 + st_of(3));
          }
        }
      }
      return v;
    };
    float4 carry1 = load_carry(kNG - 1, cs_g);
    cs_g -= cs_step;
    float4 carry2 = load_carry(kNG - 2, cs_g);
    // dB/dC accumulator row of this lane's flush (N = 16: dB for channel bit
    // 0 clear, dC for set; state st_of(0)), at the tile's first step
    float* const acc_row = (((c & 1) != 0 ? dC_b : dB_b) + static_cast<size_t>(st_of(0)) * L) + t0;

    if (use_tma) {
      bool ok = mbar_wait_bounded(&sh.bar[s], (i >> 1) & 1, p.wait_polls);
      if (kWarps == 1 && has_z) ok = ok && mbar_wait_bounded(&sh.barP, i & 1, p.wait_polls);
      bool give_up;
      if constexpr (kWarps > 1) {
        give_up = __syncthreads_or(!ok) != 0;
      } else {
        give_up = __any_sync(0xffffffffu, !ok);
      }
      if (give_up) {
        if (tid == 0) {
          atomicOr(&g_bwd_device_error, kErrTmaTimeout);
          // let the copies in flight land before the CTA exits
          mbar_wait_bounded(&sh.bar[s], (i >> 1) & 1);
          if (kWarps == 1 && has_z) mbar_wait_bounded(&sh.barP, i & 1);
          if (i == 0 && k > k_begin) mbar_wait_bounded(&sh.bar[1], 0);
          bulk_wait_all();
        }
        return;
      }
    } else {
      // each warp stages its own channel rows, warp 0 the B and C rows
      const size_t wrow = row0 + wc0;
      const int wo = wc0 * kBT;
      stage_tile_plain(bD + wo, static_cast<const T*>(p.delta), wrow, n_wch, kCPW, L, t0, lane, n_rows);
      stage_tile_plain(bU + wo, static_cast<const T*>(p.u), wrow, n_wch, kCPW, L, t0, lane, n_rows);
      stage_tile_plain(bY + wo, static_cast<const T*>(p.dout), wrow, n_wch, kCPW, L, t0, lane, n_rows);
      if (has_z) {
        stage_tile_plain(bZ + wo, static_cast<const T*>(p.z), wrow, n_wch, kCPW, L, t0, lane, n_rows);
        stage_tile_plain(bP + wo, static_cast<const T*>(p.out_pre), wrow, n_wch, kCPW, L, t0,
                         lane, n_rows);
      }
      if (warp == 0) {
        const size_t brow = static_cast<size_t>(b) * NS;
        stage_tile_plain(&sh.rawB[s][0][0], p.B32, brow, NS, NS, L, t0, lane, n_bc);
        stage_tile_plain(&sh.rawC[s][0][0], p.C32, brow, NS, NS, L, t0, lane, n_bc);
      }
      __syncwarp();
    }

    // ---- 1. transform: lane (c, q) takes steps [q * kBT / kLPC, ...) of channel c.
    // A full tile (every channel of the CTA live, every step valid, 16-byte
    // aligned accumulator rows) runs this and the group walk without the
    // per-element and per-group validity tests.
    const bool full = n_ch == kCh && t0 + kBT <= len && acc_aligned;
    auto transform = [&](auto full_t) {
      constexpr bool kFull = decltype(full_t)::value;
      constexpr int kQ = kBT / 4 / kLPC;
#pragma unroll
      for (int qq = 0; qq < kQ; ++qq) {
        const int tt = (q * kQ + qq) * 4;
        const float4 x4 = ld4s(bD, c, tt);
        const float4 u4 = ld4s(bU, c, tt);
        const float4 y4 = ld4s(bY, c, tt);
        float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f), p4 = z4;
        if (has_z) {
          z4 = ld4s(bZ, c, tt);
          p4 = ld4s(bP, c, tt);
        }
        const float xs[4] = {x4.x, x4.y, x4.z, x4.w};
        const float us[4] = {u4.x, u4.y, u4.z, u4.w};
        const float ys[4] = {y4.x, y4.y, y4.z, y4.w};
        const float zs[4] = {z4.x, z4.y, z4.z, z4.w};
        const float ps[4] = {p4.x, p4.y, p4.z, p4.w};
        float dl[4], dy[4], dz[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const bool valid = kFull || (act && t0 + tt + e < len);
          float xe = xs[e] + bias;
          if (softplus_on) xe = softplus_f(xe);
          float ye = ys[e], ze = 0.f;
          if (has_z) {
            const float sz = sigmoid_f(zs[e]);
            ze = ye * ps[e] * sz * fmaf(zs[e], 1.f - sz, 1.f);
            ye *= zs[e] * sz;
          }
          dl[e] = valid ? xe : 0.f;
          dy[e] = valid ? ye : 0.f;
          dz[e] = valid ? ze : 0.f;
          dD_acc = fmaf(dy[e], valid ? us[e] : 0.f, dD_acc);
        }
        st4s(wD, c, tt, make_float4(dl[0], dl[1], dl[2], dl[3]));
        st4s(wY, c, tt, make_float4(dy[0], dy[1], dy[2], dy[3]));
        if (has_z) st4s(bZ, c, tt, make_float4(dz[0], dz[1], dz[2], dz[3]));
      }
    };
    if (full) {
      transform(std::true_type{});
    } else {
      transform(std::false_type{});
    }
    if constexpr (kWarps > 1) {
      // the CTA's barrier of the tile: past it every warp is done with
      // position i - 1 (and, staged by plain loads, warp 0's B and C rows of
      // this position are visible); its du / ddelta / dz rows, written by
      // all threads (generic proxy), leave by TMA stores (async proxy)
      fence_proxy_async_smem();
      __syncthreads();
      if (use_tma && tid == 0) {
        if (i >= 1 && tma_store) store_pos(i - 1);
        if (k > k_begin && i >= 1) {
          bulk_wait_read_all();  // the stores have read buffer s ^ 1
          issue(i + 1);
        }
      }
    } else {
      __syncwarp();
      if (use_tma && lane == 0 && k > k_begin) {
        fence_proxy_async_smem();  // the warp's reads of rawP are done
        if (has_z) issue_pre(i + 1);
        // the other buffer held the previous position's du/ddelta/dz for its
        // bulk stores; once they have read it, refill it with position i + 1
        if (i >= 1) {
          bulk_wait_read_all();
          issue(i + 1);
        }
      }
    }

    // this lane's rows: channel c of the work rows and of u, states st_of(j)
    // of B and C
    float* const rD = wD + c * kBT;
    float* const rY = wY + c * kBT;
    T* const rU = bU + c * kBT;
    T* const rDo = bD + c * kBT;  // ddelta out (in place of delta)
    const int kW = row_key(wD, c), kU = row_key(bU, c);
    const float* rB[kS];
    int kB[kS];
#pragma unroll
    for (int j = 0; j < kS; ++j) {
      rB[j] = bB + st_of(j) * kBT;
      kB[j] = row_key(bB, st_of(j));
    }
    constexpr int kCfromB = Sh::kNSP * 2 * kBT;  // rawC[s] - rawB[s], elements
    static_assert(offsetof(Sh, rawC) - offsetof(Sh, rawB) == kCfromB * sizeof(float), "B/C");

    // delta_eff and delta_eff u (ZOH: u) of group g; delta_eff is zero past
    // the end, so delta_eff u is too (ZOH: b_bar = expm1(0) / A = 0)
    auto load_dl_du = [&](int g, float2 (&dlp)[2], float2 (&dup_)[2]) {
      const float4 dl4 = ld4p(rD + grp_off(rD, kW, g));
      const float4 u4 = ld4p(rU + grp_off(rU, kU, g));
      dlp[0] = make_float2(dl4.x, dl4.y);
      dlp[1] = make_float2(dl4.z, dl4.w);
      dup_[0] = make_float2(u4.x, u4.y);
      dup_[1] = make_float2(u4.z, u4.w);
      if constexpr (!kZOH) {
        dup_[0] = mul2(dup_[0], dlp[0]);
        dup_[1] = mul2(dup_[1], dlp[1]);
      }
    };

    // ---- 3. groups in reverse
    auto groups = [&](auto full_t) {
      constexpr bool kFull = decltype(full_t)::value;
      // two-warp CTAs walk the groups one at a time: at 2 they spilled 16 bytes
      // and measured 1.2% slower
#pragma unroll (kWarps > 1 ? 1 : 2)
    for (int g = kNG - 1; g >= 0; --g) {
      const int tg = g * kGrp;
      const float4 hcur = carry1;
      carry1 = carry2;
      if (g >= 2) {
        cs_g -= cs_step;
        carry2 = load_carry(g - 2, cs_g);
      }
      float2 dlp[2], dup_[2];
      load_dl_du(g, dlp, dup_);
      const float4 dy4 = ld4p(rY + grp_off(rY, kW, g));
      const float2 dyp[2] = {make_float2(dy4.x, dy4.y), make_float2(dy4.z, dy4.w)};
      float2 gA[2], gB[2];  // sum_n g a h_{t-1} A, sum_n g B (ZOH: g b_bar); set by slot 0
      float4 dBq[kS], dCq[kS];
#pragma unroll
      for (int j = 0; j < kS; ++j) {
        const int n = st_of(j);
        const int ob = grp_off(rB[j], kB[j], g);
        const float4 B4 = ld4p(rB[j] + ob);
        const float4 C4 = ld4p(rB[j] + kCfromB + ob);
        const float2 Bp[2] = {make_float2(B4.x, B4.y), make_float2(B4.z, B4.w)};
        const float2 Cp[2] = {make_float2(C4.x, C4.y), make_float2(C4.z, C4.w)};
        const float2 a2p = dup2(a2[j]);
        // recompute a_t and h_t over the group
        float2 ab[2], hv[2], bu[2], bb[2];
        float hh = j == 0 ? hcur.x : j == 1 ? hcur.y : j == 2 ? hcur.z : hcur.w;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float2 arg = mul2(dlp[e], a2p);
          ab[e] = make_float2(ex2(arg.x), ex2(arg.y));
          if constexpr (kZOH) {
            const float inv = 1.f / Av[j];
            bb[e].x = expm1f(dlp[e].x * Av[j]) * inv;
            bb[e].y = expm1f(dlp[e].y * Av[j]) * inv;
            bu[e] = mul2(mul2(Bp[e], bb[e]), dup_[e]);
          } else {
            bu[e] = mul2(Bp[e], dup_[e]);
          }
          hv[e].x = hh = fmaf(ab[e].x, hh, bu[e].x);
          hv[e].y = hh = fmaf(ab[e].y, hh, bu[e].y);
        }
        // adjoint, latest step first
        const float2 e0 = mul2(dyp[0], Cp[0]), e1 = mul2(dyp[1], Cp[1]);
        float2 gv[2];
        gv[1].y = fmaf(an[j], gn[j], e1.y);
        gv[1].x = fmaf(ab[1].y, gv[1].y, e1.x);
        gv[0].y = fmaf(ab[1].x, gv[1].x, e0.y);
        gv[0].x = fmaf(ab[0].y, gv[0].y, e0.x);
        gn[j] = gv[0].x;
        an[j] = ab[0].x;
        float2 dBv[2], dCv[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          // a_t h_{t-1} = h_t - b_t
          const float2 ah = add2(hv[e], make_float2(-bu[e].x, -bu[e].y));
          const float2 w = mul2(gv[e], ah);
          gA[e] = j == 0 ? mul2(w, dup2(Av[j])) : fma2(w, dup2(Av[j]), gA[e]);
          dAacc[j] = fma2(w, dlp[e], dAacc[j]);
          if constexpr (kZOH) {
            // d b_t/d delta = a_t B u, d b_t/d A = B u (delta a_t - b_bar) / A
            const float2 gBu = mul2(gv[e], mul2(Bp[e], dup_[e]));
            gA[e] = fma2(gBu, ab[e], gA[e]);
            const float inv = 1.f / Av[j];
            dAacc[j].x += gBu.x * (dlp[e].x * ab[e].x - bb[e].x) * inv;
            dAacc[j].y += gBu.y * (dlp[e].y * ab[e].y - bb[e].y) * inv;
            gB[e] = j == 0 ? mul2(gv[e], mul2(Bp[e], bb[e]))
                           : fma2(gv[e], mul2(Bp[e], bb[e]), gB[e]);
            dBv[e] = mul2(gv[e], mul2(bb[e], dup_[e]));
          } else {
            gB[e] = j == 0 ? mul2(gv[e], Bp[e]) : fma2(gv[e], Bp[e], gB[e]);
            dBv[e] = mul2(gv[e], dup_[e]);
          }
          dCv[e] = mul2(dyp[e], hv[e]);
        }
        dBq[j] = make_float4(dBv[0].x, dBv[0].y, dBv[1].x, dBv[1].y);
        dCq[j] = make_float4(dCv[0].x, dCv[0].y, dCv[1].x, dCv[1].y);
        if constexpr (kShflFlush) {
          // level 1 (channel bit 2): slots 2, 3 go to the partner, whose
          // slots 0, 1 hold the same states
          if (j >= 2) {
            add_xor4(dBq[j - 2], dBq[j], 16);
            add_xor4(dCq[j - 2], dCq[j], 16);
          }
        } else {
          sh.part[c][n ^ Cfg::part_swz(c)] = dBq[j];
        }
      }

      // sum gA, gB over the channel's lanes (reduce-scatter: lane q keeps
      // the steps it emits), then du and ddelta for those steps
      const float fa[4] = {gA[0].x, gA[0].y, gA[1].x, gA[1].y};
      const float fb[4] = {gB[0].x, gB[0].y, gB[1].x, gB[1].y};
      const int owd = grp_off(rD, kW, g), owu = grp_off(rU, kU, g);
      auto emit = [&](int e, float sa, float sb) {
        const int tl = tg + e;
        const bool valid = kFull || (act && t0 + tl < len);
        const float dlv = rD[owd + e];
        const float dyv = rY[owd + e];
        const float uv = to_f32(rU[owu + e]);
        float gd = kZOH ? sa : fmaf(uv, sb, sa);
        if (softplus_on) gd *= sigmoid_from_softplus(dlv);
        const float du = fmaf(Dv, dyv, kZOH ? sb : dlv * sb);
        gd = valid ? gd : 0.f;
        dbias_acc += gd;
        rU[owu + e] = static_cast<T>(valid ? du : 0.f);
        rDo[owu + e] = static_cast<T>(gd);
      };
      if constexpr (kLPC == 4) {
        const bool hi2 = (q & 2) != 0;
        float ka0 = hi2 ? fa[2] : fa[0], ka1 = hi2 ? fa[3] : fa[1];
        float kb0 = hi2 ? fb[2] : fb[0], kb1 = hi2 ? fb[3] : fb[1];
        ka0 += __shfl_xor_sync(0xffffffffu, hi2 ? fa[0] : fa[2], 2);
        ka1 += __shfl_xor_sync(0xffffffffu, hi2 ? fa[1] : fa[3], 2);
        kb0 += __shfl_xor_sync(0xffffffffu, hi2 ? fb[0] : fb[2], 2);
        kb1 += __shfl_xor_sync(0xffffffffu, hi2 ? fb[1] : fb[3], 2);
        const bool hi1 = (q & 1) != 0;
        float ka = hi1 ? ka1 : ka0, kb = hi1 ? kb1 : kb0;
        ka += __shfl_xor_sync(0xffffffffu, hi1 ? ka0 : ka1, 1);
        kb += __shfl_xor_sync(0xffffffffu, hi1 ? kb0 : kb1, 1);
        emit(q, ka, kb);
      } else if constexpr (kLPC == 2) {
        const bool hi = (q & 1) != 0;
        float ka0 = hi ? fa[2] : fa[0], ka1 = hi ? fa[3] : fa[1];
        float kb0 = hi ? fb[2] : fb[0], kb1 = hi ? fb[3] : fb[1];
        ka0 += __shfl_xor_sync(0xffffffffu, hi ? fa[0] : fa[2], 1);
        ka1 += __shfl_xor_sync(0xffffffffu, hi ? fa[1] : fa[3], 1);
        kb0 += __shfl_xor_sync(0xffffffffu, hi ? fb[0] : fb[2], 1);
        kb1 += __shfl_xor_sync(0xffffffffu, hi ? fb[1] : fb[3], 1);
        emit(2 * q, ka0, kb0);
        emit(2 * q + 1, ka1, kb1);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) emit(e, fa[e], fb[e]);
      }

      // dB and dC of the group: sum the channels, add into the accumulators
      const bool live = kFull || t0 + tg < len;  // warp-uniform
      const bool whole = kFull || (t0 + tg + kGrp <= len && acc_aligned);
      if constexpr (kShflFlush) {
        // level 2 (channel bit 1): slot 1 to the partner; level 3 (bit 0):
        // lanes with bit 0 clear keep dB, the others dC, of state st_of(0)
        add_xor4(dBq[0], dBq[1], 8);
        add_xor4(dCq[0], dCq[1], 8);
        const bool b0 = (c & 1) != 0;
        float4 keep = b0 ? dCq[0] : dBq[0];
        add_xor4(keep, b0 ? dBq[0] : dCq[0], 4);
        // (bounds build) the group's first and last step in this batch's NS x L slice
        MSS_BOUNDS_ONLY(const long long gsl = static_cast<long long>(st_of(0)) * L + t0 + tg;
                        const long long gsl_end = gsl + (whole ? 3 : min(3, len - 1 - t0 - tg));)
        if (live MSS_AND(in_bounds(gsl, static_cast<long long>(NS) * L, kSiteDBC) &&
                         in_bounds(gsl_end, static_cast<long long>(NS) * L, kSiteDBC))) {
          float* gp = acc_row + tg;
          if (whole) {
            if (det) {
              *reinterpret_cast<float4*>(gp) = keep;
            } else {
              atomicAdd(reinterpret_cast<float4*>(gp), keep);
            }
          } else {
            const float e4[4] = {keep.x, keep.y, keep.z, keep.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              if (t0 + tg + e < len) {
                if (det) {
                  gp[e] = e4[e];
                } else {
                  atomicAdd(gp + e, e4[e]);
                }
              }
            }
          }
        }
      } else {
        __syncwarp();
        if (live) flush_part<NS>(sh.part, dB_b, L, t0 + tg, len, whole, lane, det);
        __syncwarp();
#pragma unroll
        for (int j = 0; j < kS; ++j) {
          const int n = st_of(j);
          sh.part[c][n ^ Cfg::part_swz(c)] = dCq[j];
        }
        __syncwarp();
        if (live) flush_part<NS>(sh.part, dC_b, L, t0 + tg, len, whole, lane, det);
        __syncwarp();
      }
    }
    };
    if (full) {
      groups(std::true_type{});
    } else {
      groups(std::false_type{});
    }

    // ---- 4. the tile's du, ddelta, dz (multi-warp CTAs with TMA stores:
    // thread 0 stores them past the next tile's barrier, or below)
    if (tma_store) {
      if constexpr (kWarps == 1) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 MSS_AND(in_bounds(t0, L, kSiteTmaStore) &&
                              in_bounds(rc + kCh - 1, n_bd, kSiteTmaStore))) {
          tma_store_2d(&maps.du, t0, rc, bU);
          tma_store_2d(&maps.dd, t0, rc, bD);
          if (has_z) tma_store_2d(&maps.dz, t0, rc, bZ);
          bulk_commit();
        }
      }
    } else {
      const size_t wrow = row0 + wc0;
      const int wo = wc0 * kBT;
      unstage_tile_plain(static_cast<T*>(p.du), bU + wo, wrow, n_wch, L, t0, lane, n_rows);
      unstage_tile_plain(static_cast<T*>(p.ddelta), bD + wo, wrow, n_wch, L, t0, lane, n_rows);
      if (has_z) unstage_tile_plain(static_cast<T*>(p.dz), bZ + wo, wrow, n_wch, L, t0, lane, n_rows);
      __syncwarp();
    }
  }
  if constexpr (kWarps > 1) {
    // the last position's rows
    if (tma_store && k_last >= k_begin) {
      fence_proxy_async_smem();
      __syncthreads();
      if (tid == 0) store_pos(k_last - k_begin);
    }
  }
  if (use_tma && tid == 0) bulk_wait_all();

  // ---- per-row results
#pragma unroll
  for (int m = 1; m < kLPC; m <<= 1) {
    dD_acc += __shfl_xor_sync(0xffffffffu, dD_acc, m);
    dbias_acc += __shfl_xor_sync(0xffffffffu, dbias_acc, m);
  }
  // partial sums of this (segment, batch, channel)
  const size_t prow = static_cast<size_t>(seg) * p.batch * p.dim + row;
  if (act) {
#pragma unroll
    for (int j = 0; j < kS; ++j) {
      const int n = st_of(j);
      MSS_IF(in_bounds(prow * NS + n, n_seg * n_bd * NS, kSiteDARow))
      p.dA_part[prow * NS + n] = dAacc[j].x + dAacc[j].y;
      if (p.dh0 && seg == 0 MSS_AND(in_bounds(row * NS + n, n_bd * NS, kSiteDh0)))
        p.dh0[row * NS + n] = an[j] * gn[j];
    }
    if (q == 0 MSS_AND(in_bounds(prow, n_seg * n_bd, kSiteDDRow))) {
      p.dD_part[prow] = dD_acc;
      p.dbias_part[prow] = dbias_acc;
    }
  }
}


// Adjoint pass of a segmented backward. For segment s = blockIdx.z + 1 it
// runs g_t = dy_t C_t + a_{t+1} g_{t+1} over the segment from g = 0 past its
// end, and writes the carry a_t0 g_t0 that the segment passes to its left
// neighbour in that case (seg_G) and its sum of delta_eff (seg_dsum); the
// carry with a nonzero right seed X is seg_G + 2^(A log2 e dsum) X. Same
// lanes, staging (delta, dout, z and C only) and transform as the main pass.
template <int NS, typename T>
__global__ void __launch_bounds__(32)
    ss_bwd_segadj_kernel(const BwdParams p, const __grid_constant__ TileMaps maps) {
  using Cfg = TileCfg<NS>;
  using Sh = TileShared<NS, T>;
  constexpr int kS = Cfg::kS;
  constexpr int kLPC = Cfg::kLPC;
  constexpr int kCh = Cfg::kCh;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  Sh& sh = *reinterpret_cast<Sh*>(smem_raw);

  const int lane = threadIdx.x;
  const int b = blockIdx.y;
  const int d0 = blockIdx.x * kCh;
  const int L = p.seqlen;
  const int n_ch = min(kCh, p.dim - d0);
  const int c = lane / kLPC;
  const int q = lane % kLPC;
  const bool act = c < n_ch;
  const int d = d0 + (act ? c : 0);
  const size_t row = static_cast<size_t>(b) * p.dim + d;
  const size_t row0 = static_cast<size_t>(b) * p.dim + d0;
  const int perm = state_perm<NS>(c);
  auto st_of = [&](int j) { return q + kLPC * (j ^ perm); };

  int len = L;
  if (p.seq_lens MSS_AND(in_bounds(b, p.batch, kSiteSeqLens)))
    len = max(0, min(L, p.seq_lens[b]));
  const long long n_bd = static_cast<long long>(p.batch) * p.dim;
  const long long n_rows = n_bd * L, n_bc = static_cast<long long>(p.batch) * NS * L;
  const int seg = blockIdx.z + 1;
  const size_t seg_row = row * p.n_seg + seg;
  const int k_begin = seg * p.seg_tiles;
  const int k_end = min((L + kBT - 1) / kBT, k_begin + p.seg_tiles);
  const int k_last = len > 0 ? min((len - 1) / kBT, k_end - 1) : k_begin - 1;
  const bool use_tma = p.tma_ok != 0;
  const bool has_z = p.z != nullptr;

  float a2[kS];
#pragma unroll
  for (int j = 0; j < kS; ++j)
    a2[j] = MSS_SEL(in_bounds(d * NS + st_of(j), static_cast<long long>(p.dim) * NS, kSiteA),
                    __ldg(p.A + d * NS + st_of(j)), 0.f) * kLog2e;
  const float bias =
      p.delta_bias MSS_AND(in_bounds(d, p.dim, kSiteBias)) ? __ldg(p.delta_bias + d) : 0.f;

  constexpr uint32_t kChBytes = kCh * kBT * sizeof(T);
  constexpr uint32_t kNBytes = NS * kBT * sizeof(float);
  const int rc = static_cast<int>(row0);
  auto issue = [&](int i) {  // one thread: position i = tile k_last - i
    const int s = i & 1;
    const int x = (k_last - i) * kBT;
    uint64_t* bar = &sh.bar[s];
    mbar_arrive_expect_tx(bar, (has_z ? 3u : 2u) * kChBytes + kNBytes);
    tma_load_2d(&sh.rawD[s][0][0], &maps.d, x, rc, bar);
    tma_load_2d(&sh.rawY[s][0][0], &maps.y, x, rc, bar);
    if (has_z) tma_load_2d(&sh.rawZ[s][0][0], &maps.z, x, rc, bar);
    tma_load_2d(&sh.rawC[s][0][0], &maps.c, x, b * NS, bar);
  };
  if (use_tma && lane == 0) {
    mbar_init(&sh.bar[0], 1);
    mbar_init(&sh.bar[1], 1);
    fence_mbar_init();
    if (k_last >= k_begin) issue(0);
  }
  __syncwarp();

  float G[kS];  // a_t g_t of the step just processed (0 past the segment end)
#pragma unroll
  for (int j = 0; j < kS; ++j) G[j] = 0.f;
  float dsum = 0.f;

  for (int k = k_last; k >= k_begin; --k) {
    const int i = k_last - k;
    const int s = i & 1;
    const int t0 = k * kBT;
    T* bD = &sh.rawD[s][0][0];
    T* bY = &sh.rawY[s][0][0];
    T* bZ = &sh.rawZ[s][0][0];
    const float* bC = &sh.rawC[s][0][0];
    float* wD = Sh::kInPlace ? reinterpret_cast<float*>(bD) : &sh.wD[0][0];
    float* wY = Sh::kInPlace ? reinterpret_cast<float*>(bY) : &sh.wY[0][0];
    if (use_tma) {
      if (lane == 0 && k > k_begin) {
        fence_proxy_async_smem();  // the warp is done with the other buffer
        issue(i + 1);
      }
      const bool ok = mbar_wait_bounded(&sh.bar[s], (i >> 1) & 1, p.wait_polls);
      if (__any_sync(0xffffffffu, !ok)) {
        if (lane == 0) {
          atomicOr(&g_bwd_device_error, kErrTmaTimeout);
          mbar_wait_bounded(&sh.bar[s], (i >> 1) & 1);
          if (k > k_begin) mbar_wait_bounded(&sh.bar[s ^ 1], ((i + 1) >> 1) & 1);
        }
        return;
      }
    } else {
      stage_tile_plain(bD, static_cast<const T*>(p.delta), row0, n_ch, kCh, L, t0, lane, n_rows);
      stage_tile_plain(bY, static_cast<const T*>(p.dout), row0, n_ch, kCh, L, t0, lane, n_rows);
      if (has_z)
        stage_tile_plain(bZ, static_cast<const T*>(p.z), row0, n_ch, kCh, L, t0, lane, n_rows);
      stage_tile_plain(&sh.rawC[s][0][0], static_cast<const float*>(p.C32),
                           static_cast<size_t>(b) * NS, NS, NS, L, t0, lane, n_bc);
      __syncwarp();
    }

    // transform: delta_eff and dy = dout silu(z), zero past the end
    {
      constexpr int kQ = kBT / 4 / kLPC;
#pragma unroll
      for (int qq = 0; qq < kQ; ++qq) {
        const int tt = (q * kQ + qq) * 4;
        const float4 x4 = ld4s(bD, c, tt);
        const float4 y4 = ld4s(bY, c, tt);
        float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (has_z) z4 = ld4s(bZ, c, tt);
        const float xs[4] = {x4.x, x4.y, x4.z, x4.w};
        const float ys[4] = {y4.x, y4.y, y4.z, y4.w};
        const float zs[4] = {z4.x, z4.y, z4.z, z4.w};
        float dl[4], dy[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const bool valid = act && t0 + tt + e < len;
          float xe = xs[e] + bias;
          if (p.delta_softplus) xe = softplus_f(xe);
          float ye = ys[e];
          if (has_z) ye *= silu_f(zs[e]);
          dl[e] = valid ? xe : 0.f;
          dy[e] = valid ? ye : 0.f;
        }
        st4s(wD, c, tt, make_float4(dl[0], dl[1], dl[2], dl[3]));
        st4s(wY, c, tt, make_float4(dy[0], dy[1], dy[2], dy[3]));
      }
    }
    __syncwarp();

    const float* rD = wD + c * kBT;
    const float* rY = wY + c * kBT;
    const int kW = row_key(wD, c);
    const float* rC[kS];
    int kC[kS];
#pragma unroll
    for (int j = 0; j < kS; ++j) {
      rC[j] = bC + st_of(j) * kBT;
      kC[j] = row_key(bC, st_of(j));
    }
#pragma unroll 2
    for (int g = kNG - 1; g >= 0; --g) {
      const int ow = grp_off(rD, kW, g);
      const float4 dl4 = ld4p(rD + ow);
      const float4 dy4 = ld4p(rY + ow);
      dsum += (dl4.x + dl4.y) + (dl4.z + dl4.w);
      const float2 dlp[2] = {make_float2(dl4.x, dl4.y), make_float2(dl4.z, dl4.w)};
      const float2 dyp[2] = {make_float2(dy4.x, dy4.y), make_float2(dy4.z, dy4.w)};
#pragma unroll
      for (int j = 0; j < kS; ++j) {
        const float4 C4 = ld4p(rC[j] + grp_off(rC[j], kC[j], g));
        const float2 e0 = mul2(dyp[0], make_float2(C4.x, C4.y));
        const float2 e1 = mul2(dyp[1], make_float2(C4.z, C4.w));
        const float2 a0 = mul2(dlp[0], dup2(a2[j])), a1 = mul2(dlp[1], dup2(a2[j]));
        // latest step first: g_t = e_t + G, then G = a_t g_t
        float gg = G[j];
        gg = ex2(a1.y) * (e1.y + gg);
        gg = ex2(a1.x) * (e1.x + gg);
        gg = ex2(a0.y) * (e0.y + gg);
        gg = ex2(a0.x) * (e0.x + gg);
        G[j] = gg;
      }
    }
    __syncwarp();  // the other buffer is refilled next
  }
  if (act) {
#pragma unroll
    for (int j = 0; j < kS; ++j)
      MSS_IF(in_bounds(seg_row * NS + st_of(j), n_bd * p.n_seg * NS, kSiteSegG))
      p.seg_G[seg_row * NS + st_of(j)] = G[j];
    if (q == 0 MSS_AND(in_bounds(seg_row, n_bd * p.n_seg, kSiteSegDsum))) p.seg_dsum[seg_row] = dsum;
  }
}

// Seeds of the backward's segments, right to left: segment n_seg - 1 starts
// from dlast, segment s - 1 from seg_G(s) + 2^(A log2 e dsum(s)) seed(s).
// One thread per (batch, channel, state).
__global__ void seg_combine_bwd_kernel(const float* __restrict__ A, const float* __restrict__ dlast,
                                       const float* __restrict__ seg_G,
                                       const float* __restrict__ seg_dsum, float* seg_carry,
                                       int batch, int dim, int dstate, int n_seg) {
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i >= static_cast<long long>(batch) * dim * dstate) return;
  const int n = static_cast<int>(i % dstate);
  const long long bd = i / dstate;
  const int d = static_cast<int>(bd % dim);
  const float a2 = A[static_cast<size_t>(d) * dstate + n] * kLog2e;
  float x = dlast ? dlast[i] : 0.f;
  for (int s = n_seg - 1; s >= 0; --s) {
    const size_t sr = static_cast<size_t>(bd) * n_seg + s;
    seg_carry[sr * dstate + n] = x;
    if (s > 0) x = fmaf(exp2f(a2 * seg_dsum[sr]), x, seg_G[sr * dstate + n]);
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

cudaError_t launch_param_reduce(const float* dA_part, const float* dD_part,
                                const float* dbias_part, float* dA, float* dD, float* dbias,
                                int batch, int dim, int dstate, cudaStream_t stream) {
  const int total = dim * dstate + 2 * dim;
  reduce_params_kernel<<<(total + 255) / 256, 256, 0, stream>>>(dA_part, dD_part, dbias_part,
                                                                dA, dD, dbias, batch, dim, dstate);
  return cudaPeekAtLastError();
}

// Deterministic mode: dB and dC of (batch, dstate, step) as the sum of the
// warp columns' partials in column order (zero past a sequence's valid
// length, where no column wrote). One thread per output element; blockIdx.y
// picks dB (0) or dC (1).
__global__ void reduce_bc_kernel(const float* __restrict__ part,
                                 const int32_t* __restrict__ seq_lens, float* __restrict__ dB,
                                 float* __restrict__ dC, int batch, int dstate, int L,
                                 int n_cols) {
  const size_t nl = static_cast<size_t>(dstate) * L;
  const size_t total = static_cast<size_t>(batch) * nl;
  const int which = blockIdx.y;
  float* out = which == 0 ? dB : dC;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int b = static_cast<int>(i / nl);
    const size_t r = i % nl;  // state * L + t
    const int t = static_cast<int>(r % L);
    const int len = seq_lens ? max(0, min(L, seq_lens[b])) : L;
    float acc = 0.f;
    if (t < len) {
      const float* src = part + (static_cast<size_t>(b) * n_cols * 2 + which) * nl + r;
      for (int c = 0; c < n_cols; ++c) acc += src[static_cast<size_t>(c) * 2 * nl];
    }
    out[i] = acc;
  }
}

// B and C widened to fp32 for the scan kernels (bf16 I/O): blockIdx.y picks
// the array; exact (a bf16 is the upper half of an fp32).
__global__ void bf16_to_f32_pair_kernel(const __nv_bfloat16* __restrict__ B,
                                        const __nv_bfloat16* __restrict__ C,
                                        float* __restrict__ B32, float* __restrict__ C32,
                                        size_t n) {
  const __nv_bfloat16* src = blockIdx.y == 0 ? B : C;
  float* dst = blockIdx.y == 0 ? B32 : C32;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    dst[i] = __bfloat162float(src[i]);
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ src,
                                   __nv_bfloat16* __restrict__ dst, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
       i < n; i += static_cast<size_t>(gridDim.x) * blockDim.x)
    dst[i] = __float2bfloat16_rn(src[i]);
}

static cudaError_t launch_bwd_finish(const BwdParams& p, int dstate, int io_dtype,
                                     void* dB_out, void* dC_out, float* dA, float* dD,
                                     float* ddelta_bias, cudaStream_t stream);

// The scan kernel of kWarps-warp CTAs (plain, longest-first or segmented).
template <int NS, typename T, bool kZOH, int kWarps>
static cudaError_t launch_bwd_main(const BwdParams& p, const TileMaps& maps,
                                   cudaStream_t stream) {
  // the bytes in use: sizeof() would round up to the 1024-byte alignment
  using Sh = TileShared<NS, T, kWarps>;
  const size_t smem = offsetof(Sh, barP) + sizeof(uint64_t);
  auto kern = ss_bwd_tile_kernel<NS, T, kZOH, false, false, kWarps>;
  if constexpr (NS == 16 && !kZOH) {
    const bool std_call = p.delta_softplus != 0 && p.z != nullptr && p.dBC_part == nullptr;
    const bool lpt = p.seq_lens != nullptr && p.n_seg == 1 && p.batch <= kLongestFirstMax;
    if (lpt) {
      kern = std_call ? ss_bwd_tile_kernel<NS, T, kZOH, false, true, kWarps, true>
                      : ss_bwd_tile_kernel<NS, T, kZOH, false, true, kWarps>;
    } else if (std_call && p.n_seg == 1) {
      kern = ss_bwd_tile_kernel<NS, T, kZOH, false, false, kWarps, true>;
    } else if (std_call) {
      kern = ss_bwd_tile_kernel<NS, T, kZOH, true, false, kWarps, true>;
    } else if (p.n_seg > 1) {
      kern = ss_bwd_tile_kernel<NS, T, kZOH, true, false, kWarps>;
    }
  } else {
    if (p.n_seg > 1) kern = ss_bwd_tile_kernel<NS, T, kZOH, true, false, kWarps>;
  }
  cudaError_t e = cudaFuncSetAttribute(
      kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const unsigned gx = (p.dim + Sh::kCh - 1) / Sh::kCh;
  kern<<<dim3(gx, p.batch, p.n_seg), 32 * kWarps, smem, stream>>>(p, maps);
  return cudaPeekAtLastError();
}

// maps: boxes of one warp's channels (the adjoint pass); maps_w: of a
// kWarps-warp CTA's (the scan kernel; the same as maps for one warp).
template <int NS, typename T, bool kZOH>
static cudaError_t launch_bwd_tile_t(const BwdParams& p, const TileMaps& maps,
                                     const TileMaps& maps_w, int warps, cudaStream_t stream) {
  cudaError_t e = cudaSuccess;
  if (p.n_seg > 1) {
    // the segments' seeds: adjoint pass (segments 1 ..), then the combine
    using Sh = TileShared<NS, T>;
    const size_t smem = offsetof(Sh, barP) + sizeof(uint64_t);
    const unsigned gx = (p.dim + TileCfg<NS>::kCh - 1) / TileCfg<NS>::kCh;
    auto kern_adj = ss_bwd_segadj_kernel<NS, T>;
    e = cudaFuncSetAttribute(kern_adj, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    kern_adj<<<dim3(gx, p.batch, p.n_seg - 1), 32, smem, stream>>>(p, maps);
    const long long total = static_cast<long long>(p.batch) * p.dim * NS;
    seg_combine_bwd_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
        p.A, p.dlast, p.seg_G, p.seg_dsum, p.seg_carry, p.batch, p.dim, NS, p.n_seg);
  }
  if constexpr (NS == 16) {
    if (warps == 2) return launch_bwd_main<NS, T, kZOH, 2>(p, maps_w, stream);
  }
  return launch_bwd_main<NS, T, kZOH, 1>(p, maps, stream);
}

template <typename T, bool kZOH>
static cudaError_t launch_bwd_tile_n(const BwdParams& p, const TileMaps& maps,
                                     const TileMaps& maps_w, int warps, int dstate,
                                     cudaStream_t stream) {
  switch (dstate) {
    case 1: return launch_bwd_tile_t<1, T, kZOH>(p, maps, maps_w, warps, stream);
    case 2: return launch_bwd_tile_t<2, T, kZOH>(p, maps, maps_w, warps, stream);
    case 4: return launch_bwd_tile_t<4, T, kZOH>(p, maps, maps_w, warps, stream);
    case 8: return launch_bwd_tile_t<8, T, kZOH>(p, maps, maps_w, warps, stream);
    case 16: return launch_bwd_tile_t<16, T, kZOH>(p, maps, maps_w, warps, stream);
    default: return cudaErrorInvalidValue;
  }
}

static int tile_channels(int dstate) {
  switch (dstate) {
    case 1: return TileCfg<1>::kCh;
    case 2: return TileCfg<2>::kCh;
    case 4: return TileCfg<4>::kCh;
    case 8: return TileCfg<8>::kCh;
    default: return TileCfg<16>::kCh;
  }
}
static_assert(TileCfg<16>::kCh == 8 && TileCfg<8>::kCh == 16 && TileCfg<4>::kCh == 32 &&
                  TileCfg<2>::kCh == 32 && TileCfg<1>::kCh == 32 && kBT == kScanTile,
              "seg_plan's CTA count");

// A row-major (rows x L) operand in boxes of box_rows rows x kBT steps,
// 128-byte swizzle for fp32 rows, 64-byte for bf16 (TileShared's layout).
static bool encode_tile(CUtensorMap* m, const void* base, int io_dtype, uint64_t rows,
                        uint64_t L, uint32_t box_rows) {
  auto fn = tensor_map_encoder();
  if (!fn) return false;
  const size_t esize = io_dtype == MSS_BF16 ? 2 : 4;
  const cuuint64_t dims[2] = {L, rows};
  const cuuint64_t strides[1] = {L * esize};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBT), box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, io_dtype == MSS_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
            2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            io_dtype == MSS_BF16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Warps per CTA of the N = 16 scan kernel. Two-warp CTAs share the B and C
// staging, so that with bf16 I/O 16 warps per SM fit in shared memory (one-
// warp CTAs: 14); measured, they pay for their barrier per tile only there:
// configs[2] backward 3.63 -> 3.59 ms, while fp32 (configs[1]: 0.503 ->
// 0.523 ms) and time-segmented bf16 (configs[4]: 18.0 -> 18.3 ms) lose.
// MAMBA_SS_BWD_WARPS=1 or 2 forces either (tests).
static int bwd_warps(int dstate, int io_dtype, int n_seg) {
  if (dstate != 16) return 1;
  int w = io_dtype == MSS_BF16 && n_seg == 1 ? 2 : 1;
  if (const char* env = getenv("MAMBA_SS_BWD_WARPS")) w = atoi(env) == 1 ? 1 : 2;
  return w;
}

static bool encode_channel_maps(TileMaps* m, const BwdParams& p, int io_dtype, uint32_t ch) {
  const uint64_t rows = static_cast<uint64_t>(p.batch) * p.dim;
  const uint64_t L = p.seqlen;
  return encode_tile(&m->u, p.u, io_dtype, rows, L, ch) &&
         encode_tile(&m->d, p.delta, io_dtype, rows, L, ch) &&
         encode_tile(&m->y, p.dout, io_dtype, rows, L, ch) &&
         encode_tile(&m->du, p.du, io_dtype, rows, L, ch) &&
         encode_tile(&m->dd, p.ddelta, io_dtype, rows, L, ch) &&
         (!p.z || (encode_tile(&m->z, p.z, io_dtype, rows, L, ch) &&
                   encode_tile(&m->p, p.out_pre, io_dtype, rows, L, ch) &&
                   encode_tile(&m->dz, p.dz, io_dtype, rows, L, ch)));
}

static cudaError_t launch_bwd_tile(const BwdParams& p, int dstate, int io_dtype, int zoh,
                                   cudaStream_t stream) {
  BwdParams pk = p;
  TileMaps maps, maps_w;
  memset(&maps, 0, sizeof(maps));
  memset(&maps_w, 0, sizeof(maps_w));
  const int warps = bwd_warps(dstate, io_dtype, p.n_seg);
  const size_t esize = io_dtype == MSS_BF16 ? 2 : 4;
  const auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  pk.tma_ok = (p.seqlen * esize) % 16 == 0 && al16(p.B32) && al16(p.C32) && al16(p.u) &&
              al16(p.delta) && al16(p.dout) && al16(p.du) && al16(p.ddelta) &&
              (!p.z || (al16(p.z) && al16(p.dz) && al16(p.out_pre)));
  if (pk.tma_ok) {
    const uint64_t brows = static_cast<uint64_t>(p.batch) * dstate;
    const uint64_t L = p.seqlen;
    const uint32_t ch = static_cast<uint32_t>(tile_channels(dstate));
    const uint32_t ns = static_cast<uint32_t>(dstate);
    pk.tma_ok = encode_tile(&maps.b, p.B32, MSS_F32, brows, L, ns) &&
                encode_tile(&maps.c, p.C32, MSS_F32, brows, L, ns) &&
                encode_channel_maps(&maps, p, io_dtype, ch);
    if (pk.tma_ok) {
      maps_w = maps;
      if (warps > 1)
        pk.tma_ok = encode_channel_maps(&maps_w, p, io_dtype, ch * static_cast<uint32_t>(warps));
    }
  }
  if (io_dtype == MSS_BF16)
    return zoh ? launch_bwd_tile_n<__nv_bfloat16, true>(pk, maps, maps_w, warps, dstate, stream)
               : launch_bwd_tile_n<__nv_bfloat16, false>(pk, maps, maps_w, warps, dstate, stream);
  return zoh ? launch_bwd_tile_n<float, true>(pk, maps, maps_w, warps, dstate, stream)
             : launch_bwd_tile_n<float, false>(pk, maps, maps_w, warps, dstate, stream);
}

cudaError_t launch_bwd(const BwdParams& p, int dstate, int io_dtype, int zoh,
                       void* dB_out, void* dC_out, float* dA, float* dD,
                       float* ddelta_bias, cudaStream_t stream) {
  const size_t n_bnl = static_cast<size_t>(p.batch) * dstate * p.seqlen;
  cudaError_t e = cudaSuccess;
  if (!p.dBC_part) {  // deterministic mode writes every accumulator element itself
    e = cudaMemsetAsync(p.dB_acc, 0, n_bnl * sizeof(float), stream);
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(p.dC_acc, 0, n_bnl * sizeof(float), stream);
    if (e != cudaSuccess) return e;
  }

  if (io_dtype == MSS_BF16) {
    const int threads = 256;
    const unsigned blocks = static_cast<unsigned>(
        std::min<size_t>((n_bnl + threads - 1) / threads, 148 * 8));
    bf16_to_f32_pair_kernel<<<dim3(blocks, 2), threads, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(p.B), static_cast<const __nv_bfloat16*>(p.C), p.B32,
        p.C32, n_bnl);
    e = cudaPeekAtLastError();
    if (e != cudaSuccess) return e;
  }
  e = launch_bwd_tile(p, dstate, io_dtype, zoh, stream);
  if (e != cudaSuccess) return e;
  if (p.dBC_part) {
    const int threads = 256;
    const unsigned blocks = static_cast<unsigned>(
        std::min<size_t>((n_bnl + threads - 1) / threads, 148 * 16));
    reduce_bc_kernel<<<dim3(blocks, 2), threads, 0, stream>>>(
        p.dBC_part, p.seq_lens, p.dB_acc, p.dC_acc, p.batch, dstate, p.seqlen, p.n_cols);
    e = cudaPeekAtLastError();
    if (e != cudaSuccess) return e;
  }
  return launch_bwd_finish(p, dstate, io_dtype, dB_out, dC_out, dA, dD, ddelta_bias, stream);
}

// The batch reduction of the parameter gradients and (bf16 I/O) the
// fp32 -> bf16 conversion of dB/dC, after the scan kernel.
static cudaError_t launch_bwd_finish(const BwdParams& p, int dstate, int io_dtype,
                                     void* dB_out, void* dC_out, float* dA, float* dD,
                                     float* ddelta_bias, cudaStream_t stream) {
  const size_t n_bnl = static_cast<size_t>(p.batch) * dstate * p.seqlen;
  cudaError_t e = cudaSuccess;
  {
    const int total = p.dim * dstate + 2 * p.dim;
    const int threads = 256;
    const int blocks = (total + threads - 1) / threads;
    // partials are per (segment, batch): n_seg * batch rows
    reduce_params_kernel<<<blocks, threads, 0, stream>>>(
        p.dA_part, p.dD_part, p.dbias_part, dA, dD, ddelta_bias, p.batch * p.n_seg,
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

unsigned int take_bwd_device_error() {
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_bwd_device_error, sizeof(v)) != cudaSuccess) return ~0u;
  cudaMemcpyToSymbol(g_bwd_device_error, &zero, sizeof(zero));
  return v;
}

void take_bwd_bounds(unsigned long long out[4]) { take_oob_record(out); }

}  // namespace mss

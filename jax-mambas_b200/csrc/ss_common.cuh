// Shared device code of the sm_100a selective scan: parameter blocks,
// activation helpers, TMA / mbarrier wrappers and packed fp32 pairs.
//
// Work decomposition (forward and backward): the recurrence
// h_t = a_t h_{t-1} + b_t runs sequentially in time inside each lane; a lane
// owns up to 4 states of one channel, and the forward saves the state after
// every MSS_CHUNK (4) steps so that the backward can restart anywhere.
#pragma once

#include <cuda_bf16.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mamba_selective_scan.h"

namespace mss {

constexpr int kCkpt = MSS_CHUNK;  // steps per saved carry (chunk_states entry)

// N = 16: the lane that owns states q, q + 4, q + 8, q + 12 of channel slot c
// (of 8 in a CTA) keeps state q + 4 (j ^ state_perm(c)) in its slot j. Both
// kernels use this order (the backward needs it for its shuffle sums of dB and
// dC over channels), so saved carries need no reordering between them.
template <int NS>
__device__ __forceinline__ int state_perm(int c) {
  return NS == 16 ? (c >> 1) & 3 : 0;
}

// Saved carries are (batch, n_chunks, dim, dstate) fp32, time-major so that a
// warp's stores and loads of one carry index are contiguous. Inside a
// (batch, index, channel) entry the states are in lane-slot order: lane q's
// slots 0, 1, 2, ... (states q + lpc (j ^ perm), lpc lanes per channel) sit at
// q * (dstate / lpc) + 0, 1, 2, ..., one 16-byte word for 4 states.
__device__ __forceinline__ size_t carry_offset(int b, int idx, int n_chunks, int dim, int d,
                                               int dstate) {
  return ((static_cast<size_t>(b) * n_chunks + idx) * dim + d) * dstate;
}
constexpr float kLog2e = 1.4426950408889634f;

// Batch index of the CTAs in grid row y. With per-sequence valid lengths
// (right padding) a CTA's work is proportional to its sequence's valid
// length, and CTAs are dispatched in grid order, so the rows run longest
// sequence first (ties by index): the short CTAs fill the last wave instead
// of a long one setting the tail. Every lane of the calling warp must be
// present; batches beyond kLongestFirstMax keep the grid order.
constexpr int kLongestFirstMax = 128;
__device__ __forceinline__ int batch_of_row(const int32_t* seq_lens, int batch, int L, int y) {
  if (seq_lens == nullptr || batch > kLongestFirstMax) return y;
  const int lane = threadIdx.x & 31;
  for (int base = 0; base < batch; base += 32) {
    const int bb = base + lane;
    bool hit = false;
    if (bb < batch) {
      const int lb = max(0, min(L, __ldg(seq_lens + bb)));
      int rank = 0;
      for (int o = 0; o < batch; ++o) {
        const int lo = max(0, min(L, __ldg(seq_lens + o)));
        rank += (lo > lb || (lo == lb && o < bb)) ? 1 : 0;
      }
      hit = rank == y;
    }
    const unsigned m = __ballot_sync(0xffffffffu, hit);
    if (m != 0u) return base + __ffs(static_cast<int>(m)) - 1;
  }
  return y;
}

struct FwdParams {
  int batch, dim, seqlen, n_chunks;  // n_chunks: saved carries per row, ceil(L / kCkpt)
  int delta_softplus;
  int tma_ok;  // rows may be staged with TMA bulk copies (set by the launcher)
  unsigned int wait_polls;  // poll limit of the staging waits (set by the launcher)
  const void* u;
  const void* delta;
  const void* z;
  const void* B;
  const void* C;
  const float* A;
  const float* D;
  const float* delta_bias;
  const float* h0;
  const int32_t* seq_lens;
  void* out;
  void* out_pre;  // optional: y + D*u before the gate (read by the backward for dz)
  float* last_state;
  float* chunk_states;
  // time segments (n_seg > 1: see seg_plan): blockIdx.z is the segment, of
  // seg_tiles tiles. The end-state pass writes seg_end (batch, dim, n_seg,
  // dstate) and seg_dsum (batch, dim, n_seg); the main pass starts segment
  // s > 0 from seg_in (batch, dim, n_seg, dstate).
  int n_seg, seg_tiles;
  float* seg_end;
  float* seg_dsum;
  const float* seg_in;
};

struct BwdParams {
  int batch, dim, seqlen, n_chunks;
  int delta_softplus;
  int tma_ok;  // B/C may be staged with TMA (set by the launcher)
  unsigned int wait_polls;  // poll limit of the staging waits (set by the launcher)
  const void* u;
  const void* delta;
  const void* z;
  const void* B;
  const void* C;
  const float* A;
  const float* D;
  const float* delta_bias;
  const float* h0;
  const int32_t* seq_lens;
  const float* chunk_states;
  const void* out_pre;  // y + D*u saved by the forward (needed when z is given)
  const void* dout;
  const float* dlast;
  void* du;
  void* ddelta;
  void* dz;
  // B and C as fp32 (batch, dstate, L), what the scan kernels read: the
  // inputs themselves for fp32 I/O, a copy widened by the launcher for bf16
  float* B32;
  float* C32;
  // deterministic mode: per warp-column partial sums of dB and dC,
  // (batch, n_cols, 2, dstate, L) fp32, written (not added) by the scan
  // kernel and summed in a fixed order by reduce_bc_kernel; null otherwise
  float* dBC_part;
  int n_cols;      // warp columns: ceil(dim / channels per warp)
  float* dB_acc;   // fp32 (batch, dstate, L), zeroed before the launch
  float* dC_acc;
  float* dA_part;  // fp32 (n_seg, batch, dim, dstate): per-batch partial sums
  float* dD_part;  // fp32 (n_seg, batch, dim)
  float* dbias_part;
  float* dh0;
  // time segments (n_seg > 1: see seg_plan): blockIdx.z is the segment, of
  // seg_tiles tiles. The adjoint pass writes seg_G (batch, dim, n_seg,
  // dstate: the carry a_t0 g_t0 a segment passes left when nothing enters it
  // from the right) and seg_dsum; the main pass seeds segment s < n_seg - 1
  // with seg_carry (batch, dim, n_seg, dstate).
  int n_seg, seg_tiles;
  float* seg_G;
  float* seg_dsum;
  float* seg_carry;
};

// Complex selective scan (ss_cplx.cu): A, B, C, states complex64 (float2),
// u, delta, z, out, gradients of real arguments fp32; fp32 I/O only.
struct CplxParams {
  int batch, dim, seqlen, n_chunks;
  int delta_softplus;
  const float* u;
  const float* delta;
  const float* z;
  const void* A;        // (dim, dstate) complex
  const void* B;        // (batch, dstate, L) complex
  const void* C;
  const float* D;
  const float* delta_bias;
  const void* h0;       // (batch, dim, dstate) complex or null
  const int32_t* seq_lens;
  float* out;
  float* out_pre;
  void* last_state;     // complex
  void* chunk_states;   // (batch, n_chunks, dim, dstate) complex
  // backward
  const float* dout;
  const void* dlast;    // complex
  float* du;
  float* ddelta;
  float* dz;
  float* dB_acc_r;      // (batch, dstate, L) fp32 planes, zeroed by the launcher
  float* dB_acc_i;
  float* dC_acc_r;
  float* dC_acc_i;
  float* dA_part;       // (batch, dim, dstate, 2)
  float* dD_part;       // (batch, dim)
  float* dbias_part;
  void* dh0;            // complex
};

// Causal depthwise conv1d + SiLU (ss_conv.cu); rows are (batch, dim) in the
// scan's (batch, dim, L) layout.
struct ConvParams {
  int batch, dim, seqlen;
  int vec;                 // 4-step vector accesses allowed (set by the launcher)
  const void* x;           // (batch, dim, L)
  const float* weight;     // (kwidth, dim)
  const float* bias;       // (dim) or null
  const int32_t* seq_lens;
  const void* state_in;    // (batch, dim, kwidth - 1) or null: inputs before t = 0
  void* u;                 // forward: (batch, dim, L)
  void* state_out;         // forward: (batch, dim, kwidth - 1) or null
  const void* du;          // backward: gradient of u
  void* dx;                // backward: gradient of x
  void* dstate_in;         // backward: gradient of state_in, or null
  float* dw_part;          // backward: (batch, segments, kwidth, dim) partial sums
  float* db_part;          // backward: (batch, segments, dim)
};

struct StepParams {
  int batch, dim;
  int delta_softplus;
  float* state;  // (batch, dim, dstate) fp32, updated in place
  const void* u;
  const void* delta;
  const void* z;
  const void* B;
  const void* C;
  const float* A;
  const float* D;
  const float* delta_bias;
  void* out;
};

// ---------------------------------------------------------------- typed I/O
// bf16 -> fp32 is exact: the bf16 bits are the fp32's upper half, so the
// widening is a shift (low element of a pair) or a mask (high element).
__device__ __forceinline__ float bf16_bits_to_f32(unsigned short h) {
  return __uint_as_float(static_cast<uint32_t>(h) << 16);
}
__device__ __forceinline__ float4 bf16x4_to_f32(uint2 w) {
  return make_float4(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u),
                     __uint_as_float(w.y << 16), __uint_as_float(w.y & 0xffff0000u));
}

template <typename T>
struct Elem;

template <>
struct Elem<float> {
  static __device__ __forceinline__ float ld(const float* p) { return __ldg(p); }
  static __device__ __forceinline__ void st(float* p, float v) { *p = v; }
};

template <>
struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float ld(const __nv_bfloat16* p) {
    return bf16_bits_to_f32(__ldg(reinterpret_cast<const unsigned short*>(p)));
  }
  static __device__ __forceinline__ void st(__nv_bfloat16* p, float v) {
    *p = __float2bfloat16_rn(v);
  }
};

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) {
  return bf16_bits_to_f32(__bfloat16_as_ushort(v));
}

// ------------------------------------------------------------- activations
// 2^x on the special-function unit.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// log1p(t) for t in [0, 1] from the series
//   log1p(t) = 2 atanh(s) = 2 (s + s^3/3 + s^5/5 + ...),  s = t / (2 + t),
// with s <= 1/3 the terms through s^11 leave a relative error below 1e-7.
__device__ __forceinline__ float log1p_unit(float t) {
  const float s = __fdividef(t, 2.f + t);
  const float s2 = s * s;
  float q = fmaf(s2, 1.f / 11.f, 1.f / 9.f);
  q = fmaf(s2, q, 1.f / 7.f);
  q = fmaf(s2, q, 1.f / 5.f);
  q = fmaf(s2, q, 1.f / 3.f);
  q = fmaf(s2, q, 1.f);
  return 2.f * s * q;
}

// softplus(x) = max(x, 0) + log1p(exp(-|x|)), jax.nn.softplus's function
// (mamba/mamba1.py:76,165), evaluated without overflow for any x.
__device__ __forceinline__ float softplus_f(float x) {
  return fmaxf(x, 0.f) + log1p_unit(__expf(-fabsf(x)));
}

// 1 / (1 + e^-x) from one SFU exponential and one SFU reciprocal.
__device__ __forceinline__ float sigmoid_f(float x) {
  return __fdividef(1.f, 1.f + __expf(-x));
}

__device__ __forceinline__ float silu_f(float z) { return z * sigmoid_f(z); }

// sigmoid(x) from s = softplus(x): 1 - e^{-s}; for small s the series
// s (1 - s/2 (1 - s/3 (1 - s/4))) avoids the cancellation of 1 - e^{-s}.
__device__ __forceinline__ float sigmoid_from_softplus(float s) {
  const float series = s * fmaf(-0.5f * s, fmaf(-s * (1.f / 3.f), fmaf(-0.25f, s, 1.f), 1.f), 1.f);
  return s < 0.0625f ? series : 1.f - ex2(-s * kLog2e);
}

// ------------------------------------------------- TMA bulk copies, mbarriers
__device__ __forceinline__ uint32_t smem_u32(const void* ptr) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count)
               : "memory");
}

// Makes mbarrier initialisation visible to the TMA (async proxy).
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's generic-proxy shared-memory accesses before later
// async-proxy (TMA) writes to the same buffers.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// 2-D TMA tile copy global -> shared: the box at column x (innermost, a
// multiple of 16 bytes) and row y of the tensor map lands densely at dst
// (128-byte aligned); elements outside the tensor are filled with zeros and
// still counted on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 2-D TMA tile store shared -> global (elements outside the tensor are not
// written); completion is tracked by the issuing thread's bulk async-groups.
__device__ __forceinline__ void tma_store_2d(const void* tmap, int x, int y, const void* src) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
          reinterpret_cast<uint64_t>(tmap)),
      "r"(x), "r"(y), "r"(smem_u32(src))
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until every committed bulk store of this thread has finished reading
// shared memory (the buffers may then be overwritten).
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Asynchronous 4- / 8-byte global -> shared copies (cp.async): when `valid`
// is false nothing is read (src-size 0) and the shared bytes are zero-filled;
// `src` must still be a valid global address. commit_group / wait_group as
// in PTX.
__device__ __forceinline__ void cp_async4(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 8 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Waits until every committed bulk store of this thread has completed.
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for phase `parity` of `bar` to complete, giving up after a bounded
// number of polls (each try_wait suspends the thread for a short,
// hardware-defined time). Returns false on timeout.
// `polls` bounds the wait of a tile's staging (the launcher passes
// kWaitPolls unless mamba_ss_debug_set_wait_polls() lowered it); the waits
// that drain copies in flight before an early exit always use kWaitPolls.
constexpr uint32_t kWaitPolls = 1u << 22;
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint32_t polls = kWaitPolls) {
  for (uint32_t i = 0; i < polls; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// Bit set in a kernel's device error word when it gave up waiting for its
// TMA copies (see mamba_ss_take_device_error()).
constexpr unsigned int kErrTmaTimeout = 1u;

// ------------------------------------------------------- debug bounds build
// With MSS_BOUNDS_CHECK defined (the bounds library, libmamba_ss_b200_bounds.so),
// every plain global access whose index the kernels compute, and the
// coordinates of every TMA store, is checked against the extent of its array
// before it is made. An index outside [0, extent) is counted, the first one
// per compilation unit recorded (site, index, extent) in g_oob, and the
// access skipped, so that a wrong index shows up as a report on the host
// (mamba_ss_take_bounds_violations()) instead of a memory fault. Without the
// flag in_bounds() is the constant true and the checks compile away. Extents
// are in elements of the array's own type.
enum BoundsSite : int {
  kSiteSeqLens = 1, kSiteA, kSiteD, kSiteBias, kSiteH0, kSiteSegIn, kSiteCarry,
  kSiteOut, kSitePre, kSiteRowIn, kSiteBCIn, kSiteSegEnd, kSiteSegDsum, kSiteLast,
  kSiteDlast, kSiteSegCarry, kSiteDBC, kSiteDARow, kSiteDDRow, kSiteDh0, kSiteRowOut,
  kSiteTmaStore, kSiteSegG, kSiteParamOut, kSiteBCOut, kSiteSelfTest = 99
};
#ifdef MSS_BOUNDS_CHECK
// [0] count, [1] site, [2] index, [3] extent of the first violation
static __device__ unsigned long long g_oob[4];
#endif
__device__ __forceinline__ bool in_bounds(long long i, long long n, int site) {
#ifdef MSS_BOUNDS_CHECK
  if (i >= 0 && i < n) return true;
  if (atomicAdd(&g_oob[0], 1ull) == 0ull) {
    g_oob[1] = static_cast<unsigned long long>(site);
    g_oob[2] = static_cast<unsigned long long>(i);
    g_oob[3] = static_cast<unsigned long long>(n);
  }
  return false;
#else
  (void)i;
  (void)n;
  (void)site;
  return true;
#endif
}
// p lies inside the n elements that start at base
template <typename T>
__device__ __forceinline__ bool in_array(const T* p, const T* base, long long n, int site) {
  return in_bounds(static_cast<long long>(p - base), n, site);
}
// The kernels' check sites. Without MSS_BOUNDS_CHECK they expand to nothing
// (MSS_SEL to its second argument), so that the normal library is compiled
// from the same text as if no check were written:
//   MSS_IF(c) stmt;          stmt only if c (bounds build)
//   cond MSS_AND(c)          adds "&& c" to an existing condition
//   MSS_SEL(c, a, b)         c ? a : b (bounds build), a (normal build)
//   MSS_BOUNDS_ONLY(stmts)   statements of the bounds build only
#ifdef MSS_BOUNDS_CHECK
#define MSS_IF(c) if (c)
#define MSS_AND(c) && (c)
#define MSS_SEL(c, a, b) ((c) ? (a) : (b))
#define MSS_BOUNDS_ONLY(...) __VA_ARGS__
#else
#define MSS_IF(c)
#define MSS_AND(c)
#define MSS_SEL(c, a, b) (a)
#define MSS_BOUNDS_ONLY(...)
#endif
// Host side: copy this compilation unit's record into out[4] and clear it
// (all zero in a build without the checks).
static inline void take_oob_record(unsigned long long out[4]) {
  for (int i = 0; i < 4; ++i) out[i] = 0ull;
#ifdef MSS_BOUNDS_CHECK
  const unsigned long long zero[4] = {0ull, 0ull, 0ull, 0ull};
  if (cudaMemcpyFromSymbol(out, g_oob, sizeof(zero)) == cudaSuccess)
    cudaMemcpyToSymbol(g_oob, zero, sizeof(zero));
#endif
}

// ------------------------------------------------------- packed fp32 pairs
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  return __ffma2_rn(a, b, c);
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
// acc += the partner lane's (lane ^ m) v, component-wise, with packed adds.
__device__ __forceinline__ void add_xor4(float4& acc, const float4& v, int m) {
  const float2 lo = add2(make_float2(acc.x, acc.y),
                         make_float2(__shfl_xor_sync(0xffffffffu, v.x, m),
                                     __shfl_xor_sync(0xffffffffu, v.y, m)));
  const float2 hi = add2(make_float2(acc.z, acc.w),
                         make_float2(__shfl_xor_sync(0xffffffffu, v.z, m),
                                     __shfl_xor_sync(0xffffffffu, v.w, m)));
  acc = make_float4(lo.x, lo.y, hi.x, hi.y);
}
__device__ __forceinline__ float2 dup2(float a) { return make_float2(a, a); }

__device__ __forceinline__ float warp_sum32(float v) {
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) v += __shfl_xor_sync(0xffffffffu, v, s);
  return v;
}

// ------------------------------------- channel sums of per-lane (state, step)
// Backward kernels with the lane layout "kS = min(N, 4) states of one channel
// per lane, N / kS lanes per channel, one warp per CTA" sum dB / dC over the
// warp's channels through a [channel][state] shared tile of float4 (4 steps).
// The column swizzle keeps the 32 lanes' float4 writes of one state slot, and
// the flush's reads, free of bank conflicts.
template <int NS>
__device__ __forceinline__ int part_swz(int c) {
  return NS == 16 ? (c & 1) << 2 : NS == 8 ? (c & 3) << 1 : NS == 4 ? (c & 3)
                                           : NS == 2 ? (c >> 2) & 1 : 0;
}

// Sums one group's [channel][state] tile over the channels and adds state
// row n's four steps into acc_b[n * L + t] (t = the group's first step).
// Lane o + NS*h sums channels h*kS .. h*kS + kS - 1 of state o, then the
// 32/NS lanes of a state combine with xor-shuffles.
template <int NS>
__device__ __forceinline__ void flush_part(const float4 (*part)[NS], float* acc_b, int L, int t,
                                           int len, bool whole, int lane, bool store = false) {
  constexpr int kS = NS < 4 ? NS : 4;  // states per lane
  const int o = lane % NS, h = lane / NS;
  float2 lo = make_float2(0.f, 0.f), hi = lo;
#pragma unroll
  for (int i = 0; i < kS; ++i) {
    const int c = h * kS + i;
    const float4 v = part[c][o ^ part_swz<NS>(c)];
    lo = add2(lo, make_float2(v.x, v.y));
    hi = add2(hi, make_float2(v.z, v.w));
  }
#pragma unroll
  for (int m = NS; m < 32; m <<= 1) {
    lo.x += __shfl_xor_sync(0xffffffffu, lo.x, m);
    lo.y += __shfl_xor_sync(0xffffffffu, lo.y, m);
    hi.x += __shfl_xor_sync(0xffffffffu, hi.x, m);
    hi.y += __shfl_xor_sync(0xffffffffu, hi.y, m);
  }
  // state row o's steps t .. t + 3 (or up to len) of this batch's NS x L slice
  if (h == 0 MSS_AND(in_bounds(static_cast<long long>(o) * L + t,
                               static_cast<long long>(NS) * L, kSiteDBC) &&
                     in_bounds(static_cast<long long>(o) * L + t +
                                   (whole ? 3 : min(3, len - 1 - t)),
                               static_cast<long long>(NS) * L, kSiteDBC))) {
    float* gp = acc_b + static_cast<size_t>(o) * L + t;
    if (whole) {
      const float4 v4 = make_float4(lo.x, lo.y, hi.x, hi.y);
      if (store) {
        *reinterpret_cast<float4*>(gp) = v4;
      } else {
        atomicAdd(reinterpret_cast<float4*>(gp), v4);
      }
    } else {
      const float e4[4] = {lo.x, lo.y, hi.x, hi.y};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (t + e < len) {
          if (store) {
            gp[e] = e4[e];
          } else {
            atomicAdd(gp + e, e4[e]);
          }
        }
      }
    }
  }
}

}  // namespace mss

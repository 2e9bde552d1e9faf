// Causal depthwise conv1d + bias + SiLU + padding mask for sm_100a: the
// operation between the input projection and the selective scan in the
// Mamba block (mamba/mamba1.py:313-329, flax nnx.Conv with
// feature_group_count = d_inner and CAUSAL padding, mamba1.py:250-255):
//   xm_t  = x_t  (t < len, else 0; the inputs before t = 0 come from the
//           conv state: the previous call's last kwidth - 1 inputs)
//   u_t   = silu(bias + sum_k w_k xm_{t - (kwidth-1) + k})   (t < len, else 0)
// in the scan's (batch, dim, L) layout. The projections around it are GEMMs
// that produce / consume that layout through transposed operands, so no
// transpose pass remains around the scan.
//
// One warp per (batch, channel) row walks L in chunks of 128 steps (4 per
// lane, 16-byte loads); the kwidth - 1 inputs before a lane's steps come from
// the previous lane by shuffles and across chunks from a carried register.
// The backward walks the chunks right to left, carrying the gradient of the
// following steps the same way; dweight and dbias are reduced per row in
// registers and over the batch in a fixed order.
#include "ss_common.cuh"
#include "ss_launch.h"

namespace mss {

constexpr int kConvChunk = 128;  // steps per warp iteration

__device__ __forceinline__ float dsilu(float c) {
  const float s = sigmoid_f(c);
  return s * fmaf(c, 1.f - s, 1.f);
}

// Four steps t .. t+3 of a row (fp32); steps at or past `lim` read 0.
template <typename T>
__device__ __forceinline__ void load4_row(const T* row, int t, int lim, bool vec, float (&v)[4]) {
  if (vec && t + 4 <= lim) {
    if constexpr (sizeof(T) == 4) {
      const float4 f = *reinterpret_cast<const float4*>(row + t);
      v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
    } else {
      const float4 f = bf16x4_to_f32(*reinterpret_cast<const uint2*>(row + t));
      v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
    }
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = t + e < lim ? Elem<T>::ld(row + t + e) : 0.f;
  }
}

template <typename T>
__device__ __forceinline__ void store4_row(T* row, int t, int L, bool vec, const float (&v)[4]) {
  if (vec && t + 4 <= L) {
    if constexpr (sizeof(T) == 4) {
      *reinterpret_cast<float4*>(row + t) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
      uint2 w;
      *reinterpret_cast<__nv_bfloat162*>(&w.x) = __floats2bfloat162_rn(v[0], v[1]);
      *reinterpret_cast<__nv_bfloat162*>(&w.y) = __floats2bfloat162_rn(v[2], v[3]);
      *reinterpret_cast<uint2*>(row + t) = w;
    }
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (t + e < L) Elem<T>::st(row + t + e, v[e]);
  }
}

// Work units: a warp takes a segment of kConvSegChunks chunks of one row
// (unit = row * n_seg + segment), so that a layer splits into many equal
// units (no partial last wave) and each warp has all its loads in flight at
// once. Pre-segment inputs (forward) and post-segment gradients (backward)
// are read or recomputed at the segment edges.
constexpr int kConvSegChunks = 4;
constexpr int kConvSeg = kConvSegChunks * kConvChunk;  // steps per segment

// masked input t of a row (the conv state before t = 0; 0 before that)
template <typename T, int K>
__device__ __forceinline__ float conv_input(const T* xr, const T* sin, int t, int len) {
  if (t >= 0) return t < len ? Elem<T>::ld(xr + t) : 0.f;
  return (sin && t >= -(K - 1)) ? Elem<T>::ld(sin + (K - 1) + t) : 0.f;
}

template <typename T, int K>
__global__ void __launch_bounds__(128) ss_conv_fwd_kernel(const ConvParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int L = p.seqlen;
  const int n_seg = (L + kConvSeg - 1) / kConvSeg;
  const long long unit = static_cast<long long>(blockIdx.x) * 4 + warp;
  if (unit >= static_cast<long long>(p.batch) * p.dim * n_seg) return;  // warp-uniform
  const long long r = unit / n_seg;  // b * dim + d
  const int s0 = static_cast<int>(unit % n_seg) * kConvSeg;
  const int b = static_cast<int>(r / p.dim), d = static_cast<int>(r % p.dim);
  int len = L;
  if (p.seq_lens) len = max(0, min(L, p.seq_lens[b]));
  const T* __restrict__ xr = static_cast<const T*>(p.x) + r * L;
  T* __restrict__ ur = static_cast<T*>(p.u) + r * L;
  const T* sin = p.state_in ? static_cast<const T*>(p.state_in) + r * (K - 1) : nullptr;
  float w[K];
#pragma unroll
  for (int k = 0; k < K; ++k) w[k] = __ldg(p.weight + static_cast<size_t>(k) * p.dim + d);
  const float bias = p.bias ? __ldg(p.bias + d) : 0.f;

  // all of the segment's inputs first (independent loads)
  float xs[kConvSegChunks][4];
#pragma unroll
  for (int c = 0; c < kConvSegChunks; ++c)
    load4_row(xr, s0 + c * kConvChunk + lane * 4, len, p.vec != 0, xs[c]);
  // masked inputs at s0 - 3 .. s0 - 1
  float c3[3];
  {
    const float v = lane < 3 ? conv_input<T, K>(xr, sin, s0 - 3 + lane, len) : 0.f;
    c3[0] = __shfl_sync(0xffffffffu, v, 0);
    c3[1] = __shfl_sync(0xffffffffu, v, 1);
    c3[2] = __shfl_sync(0xffffffffu, v, 2);
  }
#pragma unroll
  for (int c = 0; c < kConvSegChunks; ++c) {
    const int t0 = s0 + c * kConvChunk;
    if (t0 >= L) break;  // warp-uniform
    const int t = t0 + lane * 4;
    const float(&xv)[4] = xs[c];
    float p1 = __shfl_up_sync(0xffffffffu, xv[1], 1);
    float p2 = __shfl_up_sync(0xffffffffu, xv[2], 1);
    float p3 = __shfl_up_sync(0xffffffffu, xv[3], 1);
    if (lane == 0) {
      p1 = c3[0];
      p2 = c3[1];
      p3 = c3[2];
    }
    const float win[7] = {p1, p2, p3, xv[0], xv[1], xv[2], xv[3]};
    float uv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float acc = bias;
#pragma unroll
      for (int k = 0; k < K; ++k) acc = fmaf(w[k], win[e + 4 - K + k], acc);
      uv[e] = t + e < len ? silu_f(acc) : 0.f;
    }
    store4_row(ur, t, L, p.vec != 0, uv);
    c3[0] = __shfl_sync(0xffffffffu, xv[1], 31);
    c3[1] = __shfl_sync(0xffffffffu, xv[2], 31);
    c3[2] = __shfl_sync(0xffffffffu, xv[3], 31);
  }
  // the last kwidth - 1 masked inputs: the conv state of the next call
  if (p.state_out && s0 + kConvSeg >= L && lane < K - 1)
    Elem<T>::st(static_cast<T*>(p.state_out) + r * (K - 1) + lane,
                conv_input<T, K>(xr, sin, L - (K - 1) + lane, len));
}

template <typename T, int K>
__global__ void __launch_bounds__(128) ss_conv_bwd_kernel(const ConvParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int L = p.seqlen;
  const int n_seg = (L + kConvSeg - 1) / kConvSeg;
  const long long unit = static_cast<long long>(blockIdx.x) * 4 + warp;
  if (unit >= static_cast<long long>(p.batch) * p.dim * n_seg) return;
  const long long r = unit / n_seg;
  const int seg = static_cast<int>(unit % n_seg);
  const int s0 = seg * kConvSeg, s1 = min(L, s0 + kConvSeg);
  const int b = static_cast<int>(r / p.dim), d = static_cast<int>(r % p.dim);
  int len = L;
  if (p.seq_lens) len = max(0, min(L, p.seq_lens[b]));
  const T* __restrict__ xr = static_cast<const T*>(p.x) + r * L;
  const T* __restrict__ gr = static_cast<const T*>(p.du) + r * L;
  T* __restrict__ dxr = static_cast<T*>(p.dx) + r * L;
  const T* sin = p.state_in ? static_cast<const T*>(p.state_in) + r * (K - 1) : nullptr;
  float w[K];
#pragma unroll
  for (int k = 0; k < K; ++k) w[k] = __ldg(p.weight + static_cast<size_t>(k) * p.dim + d);
  const float bias = p.bias ? __ldg(p.bias + d) : 0.f;

  float xs[kConvSegChunks][4], ds[kConvSegChunks][4];
#pragma unroll
  for (int c = 0; c < kConvSegChunks; ++c) {
    const int t = s0 + c * kConvChunk + lane * 4;
    load4_row(xr, t, len, p.vec != 0, xs[c]);
    load4_row(gr, t, len, p.vec != 0, ds[c]);
  }
  // gradient of the conv output (before SiLU) at s1 .. s1 + 2, recomputed
  float gn[3];
  {
    float v = 0.f;
    const int t = s1 + lane;
    if (lane < 3 && t < len) {
      float acc = bias;
#pragma unroll
      for (int k = 0; k < K; ++k)
        acc = fmaf(w[k], conv_input<T, K>(xr, sin, t - (K - 1) + k, len), acc);
      v = Elem<T>::ld(gr + t) * dsilu(acc);
    }
    gn[0] = __shfl_sync(0xffffffffu, v, 0);
    gn[1] = __shfl_sync(0xffffffffu, v, 1);
    gn[2] = __shfl_sync(0xffffffffu, v, 2);
  }
  float dwp[K], dbp = 0.f;
#pragma unroll
  for (int k = 0; k < K; ++k) dwp[k] = 0.f;
#pragma unroll
  for (int c = kConvSegChunks - 1; c >= 0; --c) {
    const int t0 = s0 + c * kConvChunk;
    if (t0 >= L) continue;  // warp-uniform
    const int t = t0 + lane * 4;
    const float(&xv)[4] = xs[c];
    const float(&dv)[4] = ds[c];
    float p1 = __shfl_up_sync(0xffffffffu, xv[1], 1);
    float p2 = __shfl_up_sync(0xffffffffu, xv[2], 1);
    float p3 = __shfl_up_sync(0xffffffffu, xv[3], 1);
    if (c > 0) {
      const float q1 = __shfl_sync(0xffffffffu, xs[c > 0 ? c - 1 : 0][1], 31);
      const float q2 = __shfl_sync(0xffffffffu, xs[c > 0 ? c - 1 : 0][2], 31);
      const float q3 = __shfl_sync(0xffffffffu, xs[c > 0 ? c - 1 : 0][3], 31);
      if (lane == 0) {
        p1 = q1;
        p2 = q2;
        p3 = q3;
      }
    } else {
      // the three inputs before the segment (the conv state before t = 0)
      const float v = lane < 3 ? conv_input<T, K>(xr, sin, s0 - 3 + lane, len) : 0.f;
      const float q1 = __shfl_sync(0xffffffffu, v, 0);
      const float q2 = __shfl_sync(0xffffffffu, v, 1);
      const float q3 = __shfl_sync(0xffffffffu, v, 2);
      if (lane == 0) {
        p1 = q1;
        p2 = q2;
        p3 = q3;
      }
    }
    const float win[7] = {p1, p2, p3, xv[0], xv[1], xv[2], xv[3]};
    float g[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float acc = bias;
#pragma unroll
      for (int k = 0; k < K; ++k) acc = fmaf(w[k], win[e + 4 - K + k], acc);
      g[e] = t + e < len ? dv[e] * dsilu(acc) : 0.f;
    }
    float n0 = __shfl_down_sync(0xffffffffu, g[0], 1);
    float n1 = __shfl_down_sync(0xffffffffu, g[1], 1);
    float n2 = __shfl_down_sync(0xffffffffu, g[2], 1);
    if (lane == 31) {
      n0 = gn[0];
      n1 = gn[1];
      n2 = gn[2];
    }
    const float gw[7] = {g[0], g[1], g[2], g[3], n0, n1, n2};
    float dxv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < K; ++k) acc = fmaf(w[k], gw[e + K - 1 - k], acc);
      dxv[e] = t + e < len ? acc : 0.f;
      dbp += g[e];
#pragma unroll
      for (int k = 0; k < K; ++k) dwp[k] = fmaf(g[e], win[e + 4 - K + k], dwp[k]);
    }
    store4_row(dxr, t, L, p.vec != 0, dxv);
    gn[0] = __shfl_sync(0xffffffffu, g[0], 0);
    gn[1] = __shfl_sync(0xffffffffu, g[1], 0);
    gn[2] = __shfl_sync(0xffffffffu, g[2], 0);
  }
  // gradient of the conv state: input -(K-1)+j feeds the outputs t = j - k
  if (seg == 0 && p.dstate_in && lane < K - 1) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k)
      if (k <= lane) acc = fmaf(w[k], lane - k == 0 ? gn[0] : lane - k == 1 ? gn[1] : gn[2], acc);
    Elem<T>::st(static_cast<T*>(p.dstate_in) + r * (K - 1) + lane, acc);
  }
  // per-(row, segment) partial sums of dweight and dbias
#pragma unroll
  for (int k = 0; k < K; ++k) dwp[k] = warp_sum32(dwp[k]);
  dbp = warp_sum32(dbp);
  if (lane == 0) {
    const size_t bs = static_cast<size_t>(b) * n_seg + seg;  // partial row (batch, segment)
#pragma unroll
    for (int k = 0; k < K; ++k) p.dw_part[(bs * K + k) * p.dim + d] = dwp[k];
    p.db_part[bs * p.dim + d] = dbp;
  }
}

// dweight (kwidth, dim) and dbias (dim) from the per-(batch, segment)
// partials, summed in a fixed order.
__global__ void conv_reduce_kernel(const float* __restrict__ dw_part,
                                   const float* __restrict__ db_part, float* dweight,
                                   float* dbias, int batch, int dim, int kwidth) {
  const int n = kwidth * dim;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n + dim;
       i += gridDim.x * blockDim.x) {
    float s = 0.f;
    if (i < n) {
      for (int b = 0; b < batch; ++b) s += dw_part[static_cast<size_t>(b) * n + i];
      dweight[i] = s;
    } else if (dbias) {
      for (int b = 0; b < batch; ++b) s += db_part[static_cast<size_t>(b) * dim + (i - n)];
      dbias[i - n] = s;
    }
  }
}

// One decode token of the conv (Mamba.step, mamba/mamba1.py:339-355): per
// (batch, channel), u = silu(bias + sum_k w_k [state, x]_k) over the conv
// state (the last kwidth - 1 inputs) followed by the new input x, and the
// state shifts by one (in place). One thread per (batch, channel).
template <typename T, int K>
__global__ void __launch_bounds__(256) ss_conv_step_kernel(const ConvParams p) {
  const long long r = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= static_cast<long long>(p.batch) * p.dim) return;
  const int d = static_cast<int>(r % p.dim);
  float win[K];
  T* st = static_cast<T*>(p.state_out) + r * (K - 1);
#pragma unroll
  for (int j = 0; j < K - 1; ++j) win[j] = Elem<T>::ld(st + j);
  win[K - 1] = Elem<T>::ld(static_cast<const T*>(p.x) + r);
  float acc = p.bias ? __ldg(p.bias + d) : 0.f;
#pragma unroll
  for (int k = 0; k < K; ++k) acc = fmaf(__ldg(p.weight + static_cast<size_t>(k) * p.dim + d), win[k], acc);
  Elem<T>::st(static_cast<T*>(p.u) + r, silu_f(acc));
#pragma unroll
  for (int j = 0; j < K - 1; ++j) Elem<T>::st(st + j, win[j + 1]);
}

template <typename T>
static cudaError_t launch_conv_step_t(const ConvParams& p, int kwidth, cudaStream_t stream) {
  const long long rows = static_cast<long long>(p.batch) * p.dim;
  const unsigned grid = static_cast<unsigned>((rows + 255) / 256);
  switch (kwidth) {
    case 1: ss_conv_step_kernel<T, 1><<<grid, 256, 0, stream>>>(p); break;
    case 2: ss_conv_step_kernel<T, 2><<<grid, 256, 0, stream>>>(p); break;
    case 3: ss_conv_step_kernel<T, 3><<<grid, 256, 0, stream>>>(p); break;
    case 4: ss_conv_step_kernel<T, 4><<<grid, 256, 0, stream>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaPeekAtLastError();
}

cudaError_t launch_conv_step(const ConvParams& p, int kwidth, int io_dtype, cudaStream_t stream) {
  if (io_dtype == MSS_BF16) return launch_conv_step_t<__nv_bfloat16>(p, kwidth, stream);
  return launch_conv_step_t<float>(p, kwidth, stream);
}

template <typename T>
static cudaError_t launch_conv_t(const ConvParams& p, int kwidth, bool backward,
                                 float* dweight, float* dbias, cudaStream_t stream) {
  const long long units = static_cast<long long>(p.batch) * p.dim * conv_segments(p.seqlen);
  const dim3 grid(static_cast<unsigned>((units + 3) / 4));
  switch (kwidth) {
#define MSS_CONV_CASE(KW)                                                   \
  case KW:                                                                  \
    if (backward)                                                           \
      ss_conv_bwd_kernel<T, KW><<<grid, 128, 0, stream>>>(p);               \
    else                                                                    \
      ss_conv_fwd_kernel<T, KW><<<grid, 128, 0, stream>>>(p);               \
    break;
    MSS_CONV_CASE(1)
    MSS_CONV_CASE(2)
    MSS_CONV_CASE(3)
    MSS_CONV_CASE(4)
#undef MSS_CONV_CASE
    default:
      return cudaErrorInvalidValue;
  }
  cudaError_t e = cudaPeekAtLastError();
  if (e != cudaSuccess || !backward) return e;
  const int total = kwidth * p.dim + p.dim;
  conv_reduce_kernel<<<(total + 255) / 256, 256, 0, stream>>>(
      p.dw_part, p.db_part, dweight, dbias, p.batch * conv_segments(p.seqlen), p.dim, kwidth);
  return cudaPeekAtLastError();
}

int conv_segments(int length) { return (length + kConvSeg - 1) / kConvSeg; }

cudaError_t launch_conv(const ConvParams& p_in, int kwidth, int io_dtype, bool backward,
                        float* dweight, float* dbias, cudaStream_t stream) {
  ConvParams p = p_in;
  const size_t esize = io_dtype == MSS_BF16 ? 2 : 4;
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  // 4-step vector accesses need 16-byte aligned fp32 / 8-byte aligned bf16 rows
  p.vec = (p.seqlen % 4) == 0 && al16(p.x) &&
          (backward ? (al16(p.du) && al16(p.dx)) : al16(p.u)) && (esize == 4 || esize == 2);
  if (io_dtype == MSS_BF16)
    return launch_conv_t<__nv_bfloat16>(p, kwidth, backward, dweight, dbias, stream);
  return launch_conv_t<float>(p, kwidth, backward, dweight, dbias, stream);
}

}  // namespace mss

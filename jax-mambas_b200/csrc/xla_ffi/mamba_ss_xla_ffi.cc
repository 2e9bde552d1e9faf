// XLA typed-FFI handlers over the C ABI of libmamba_ss_b200.
//
// The reference registers three handlers with jax.ffi.register_ffi_target
// (mamba/selective_scan_cuda.py:42-51): MambaSelectiveScan and
// MambaSelectiveScanBenchmark (native/selective_scan_cuda.cu:554-598) and
// MambaSelectiveScanBackward (native/selective_scan_bwd.cu:166-190). This file
// defines handlers of the same names and attribute / argument / result lists,
// each a one-to-one unpack of the typed buffers into a mamba_ss_* call, so the
// reference's Python module can load this library in place of its own.
//
// Differences a caller sees:
//  * the chunk_states residual is this library's (mamba_ss_chunk_states_elems
//    fp32 elements, any shape of that size) instead of (B, D, ceil(L/2048),
//    N, 2): the Python side's ShapeDtypeStruct for it changes accordingly;
//  * the backward takes its workspace (mamba_ss_bwd_workspace_bytes) from
//    XLA's scratch allocator.
//
// Built only by the CMake recipe with -DMAMBA_SS_XLA_FFI=ON, which needs
// jaxlib's FFI headers (jax.ffi.include_dir()).
#include <cuda_runtime.h>

#include <string>

#include "mamba_selective_scan.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

ffi::Error ToFfi(mss_status st, const char* where) {
  if (st == MSS_OK) return ffi::Error::Success();
  std::string msg = std::string(where) + ": " + mamba_ss_last_error();
  if (st == MSS_INVALID_ARGUMENT)
    return ffi::Error(ffi::ErrorCode::kInvalidArgument, msg);
  return ffi::Error(ffi::ErrorCode::kInternal, msg);
}

ffi::Error CheckResidual(size_t elems, int32_t batch, int32_t length, int32_t dim,
                         int32_t dstate) {
  const int64_t need = mamba_ss_chunk_states_elems(batch, length, dim, dstate);
  if (static_cast<int64_t>(elems) < need)
    return ffi::Error(ffi::ErrorCode::kInvalidArgument,
                      "chunk_states must hold mamba_ss_chunk_states_elems() = " +
                          std::to_string(need) + " fp32 elements, got " +
                          std::to_string(elems));
  return ffi::Error::Success();
}

ffi::Error ForwardImpl(cudaStream_t stream, int32_t discretization, int32_t batch,
                       int32_t length, int32_t dim, int32_t dstate,
                       ffi::Buffer<ffi::F32> A, ffi::Buffer<ffi::F32> deltas,
                       ffi::Buffer<ffi::F32> Bs, ffi::Buffer<ffi::F32> Cs,
                       ffi::Buffer<ffi::F32> u, ffi::Buffer<ffi::F32> initial_x,
                       ffi::ResultBuffer<ffi::F32> y, ffi::ResultBuffer<ffi::F32> final_x,
                       ffi::ResultBuffer<ffi::F32> chunk_states) {
  ffi::Error e = CheckResidual(chunk_states->element_count(), batch, length, dim, dstate);
  if (e.failure()) return e;
  return ToFfi(mamba_ss_fwd(stream, discretization, batch, length, dim, dstate,
                            A.typed_data(), deltas.typed_data(), Bs.typed_data(),
                            Cs.typed_data(), u.typed_data(), initial_x.typed_data(),
                            y->typed_data(), final_x->typed_data(),
                            chunk_states->typed_data()),
               "MambaSelectiveScan");
}

ffi::Error BenchmarkImpl(cudaStream_t stream, int32_t discretization, int32_t repeats,
                         int32_t batch, int32_t length, int32_t dim, int32_t dstate,
                         ffi::Buffer<ffi::F32> A, ffi::Buffer<ffi::F32> deltas,
                         ffi::Buffer<ffi::F32> Bs, ffi::Buffer<ffi::F32> Cs,
                         ffi::Buffer<ffi::F32> u, ffi::Buffer<ffi::F32> initial_x,
                         ffi::ResultBuffer<ffi::F32> y, ffi::ResultBuffer<ffi::F32> final_x,
                         ffi::ResultBuffer<ffi::F32> chunk_states) {
  ffi::Error e = CheckResidual(chunk_states->element_count(), batch, length, dim, dstate);
  if (e.failure()) return e;
  return ToFfi(mamba_ss_fwd_bench(stream, discretization, repeats, batch, length, dim, dstate,
                                  A.typed_data(), deltas.typed_data(), Bs.typed_data(),
                                  Cs.typed_data(), u.typed_data(), initial_x.typed_data(),
                                  y->typed_data(), final_x->typed_data(),
                                  chunk_states->typed_data()),
               "MambaSelectiveScanBenchmark");
}

ffi::Error BackwardImpl(cudaStream_t stream, ffi::ScratchAllocator scratch, int32_t batch,
                        int32_t length, int32_t dim, int32_t dstate,
                        ffi::Buffer<ffi::F32> A, ffi::Buffer<ffi::F32> deltas,
                        ffi::Buffer<ffi::F32> Bs, ffi::Buffer<ffi::F32> Cs,
                        ffi::Buffer<ffi::F32> u, ffi::Buffer<ffi::F32> initial_x,
                        ffi::Buffer<ffi::F32> chunk_states, ffi::Buffer<ffi::F32> dy,
                        ffi::Buffer<ffi::F32> dfinal_x, ffi::ResultBuffer<ffi::F32> dA,
                        ffi::ResultBuffer<ffi::F32> ddeltas, ffi::ResultBuffer<ffi::F32> dB,
                        ffi::ResultBuffer<ffi::F32> dC, ffi::ResultBuffer<ffi::F32> du,
                        ffi::ResultBuffer<ffi::F32> dinitial_x) {
  const size_t ws_bytes = mamba_ss_bwd_workspace_bytes(batch, length, dim, dstate, MSS_F32);
  auto ws = scratch.Allocate(ws_bytes, 256);
  if (!ws.has_value())
    return ffi::Error(ffi::ErrorCode::kResourceExhausted,
                      "MambaSelectiveScanBackward: no scratch for the workspace");
  // the reference's backward is Euler-only (ZOH takes JAX autodiff)
  return ToFfi(mamba_ss_bwd(stream, MSS_EULER, batch, length, dim, dstate, A.typed_data(),
                            deltas.typed_data(), Bs.typed_data(), Cs.typed_data(),
                            u.typed_data(), initial_x.typed_data(), chunk_states.typed_data(),
                            dy.typed_data(), dfinal_x.typed_data(), dA->typed_data(),
                            ddeltas->typed_data(), dB->typed_data(), dC->typed_data(),
                            du->typed_data(), dinitial_x->typed_data(), *ws, ws_bytes),
               "MambaSelectiveScanBackward");
}

}  // namespace

XLA_FFI_DEFINE_HANDLER_SYMBOL(MambaSelectiveScan, ForwardImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Attr<int32_t>("discretization")
                                  .Attr<int32_t>("batch")
                                  .Attr<int32_t>("length")
                                  .Attr<int32_t>("dim")
                                  .Attr<int32_t>("dstate")
                                  .Arg<ffi::Buffer<ffi::F32>>()   // A (D, N)
                                  .Arg<ffi::Buffer<ffi::F32>>()   // deltas, physical (B, D, L)
                                  .Arg<ffi::Buffer<ffi::F32>>()   // B, physical (B, N, L)
                                  .Arg<ffi::Buffer<ffi::F32>>()   // C, physical (B, N, L)
                                  .Arg<ffi::Buffer<ffi::F32>>()   // u, physical (B, D, L)
                                  .Arg<ffi::Buffer<ffi::F32>>()   // initial_x (B, D, N)
                                  .Ret<ffi::Buffer<ffi::F32>>()   // y, physical (B, D, L)
                                  .Ret<ffi::Buffer<ffi::F32>>()   // final_x (B, D, N)
                                  .Ret<ffi::Buffer<ffi::F32>>());  // chunk_states

XLA_FFI_DEFINE_HANDLER_SYMBOL(MambaSelectiveScanBenchmark, BenchmarkImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Attr<int32_t>("discretization")
                                  .Attr<int32_t>("repeats")
                                  .Attr<int32_t>("batch")
                                  .Attr<int32_t>("length")
                                  .Attr<int32_t>("dim")
                                  .Attr<int32_t>("dstate")
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>());

XLA_FFI_DEFINE_HANDLER_SYMBOL(MambaSelectiveScanBackward, BackwardImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Ctx<ffi::ScratchAllocator>()
                                  .Attr<int32_t>("batch")
                                  .Attr<int32_t>("length")
                                  .Attr<int32_t>("dim")
                                  .Attr<int32_t>("dstate")
                                  .Arg<ffi::Buffer<ffi::F32>>()   // A
                                  .Arg<ffi::Buffer<ffi::F32>>()   // deltas
                                  .Arg<ffi::Buffer<ffi::F32>>()   // B
                                  .Arg<ffi::Buffer<ffi::F32>>()   // C
                                  .Arg<ffi::Buffer<ffi::F32>>()   // u
                                  .Arg<ffi::Buffer<ffi::F32>>()   // initial_x
                                  .Arg<ffi::Buffer<ffi::F32>>()   // chunk_states
                                  .Arg<ffi::Buffer<ffi::F32>>()   // dy
                                  .Arg<ffi::Buffer<ffi::F32>>()   // dfinal_x
                                  .Ret<ffi::Buffer<ffi::F32>>()   // dA
                                  .Ret<ffi::Buffer<ffi::F32>>()   // ddeltas
                                  .Ret<ffi::Buffer<ffi::F32>>()   // dB
                                  .Ret<ffi::Buffer<ffi::F32>>()   // dC
                                  .Ret<ffi::Buffer<ffi::F32>>()   // du
                                  .Ret<ffi::Buffer<ffi::F32>>());  // dinitial_x

// XLA FFI handlers (typed FFI, api_version 1) over the liblp_b200 C ABI, for JAX's
// jax.ffi.ffi_call. Built only where jaxlib ships its headers (jax.ffi.include_dir()):
//   g++ -std=c++17 -O2 -shared -fPIC -I$(python -c 'import jax.ffi;print(jax.ffi.include_dir())') \
//       -I/usr/local/cuda/include lp_xla_ffi.cc -L. -llp_b200 -Wl,-rpath,'$ORIGIN' -o liblp_b200_xla.so
// (gemma4_posttrain_jax_b200.build.build_xla_ffi() runs this). The handlers only unpack
// buffers and attributes and call the C ABI on XLA's stream; the C ABI validates shapes.
// Targets: lp_fwd, lp_combine, lp_bwd (registered for platform "CUDA" by jax_ffi.py).
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "../../include/lp_logprob.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

ffi::Error status(int rc, const char* what) {
  if (rc == LP_OK) return ffi::Error::Success();
  const ffi::ErrorCode code = rc == LP_EINVAL ? ffi::ErrorCode::kInvalidArgument : ffi::ErrorCode::kInternal;
  return ffi::Error(code, std::string(what) + ": " + lp_last_error());
}

// H [T, d] bf16, W [Vs, d] bf16, y [T] s32 -> stats [3, T] f32, logp [T] f32, workspace u8
ffi::Error FwdImpl(cudaStream_t stream, ffi::Buffer<ffi::BF16> H, ffi::Buffer<ffi::BF16> W, ffi::Buffer<ffi::S32> y,
                   ffi::ResultBuffer<ffi::F32> stats, ffi::ResultBuffer<ffi::F32> logp,
                   ffi::ResultBuffer<ffi::U8> workspace, float softcap, int64_t v_off) {
  const auto hd = H.dimensions();
  const auto wd = W.dimensions();
  if (hd.size() != 2 || wd.size() != 2) return ffi::Error::InvalidArgument("lp_fwd: H and W must be rank 2");
  const int rc = lp_fwd(stream, H.untyped_data(), hd[0], hd[1], hd[1], W.untyped_data(), wd[0], v_off,
                        static_cast<const int32_t*>(y.untyped_data()), softcap,
                        static_cast<float*>(stats->untyped_data()), static_cast<float*>(logp->untyped_data()),
                        workspace->untyped_data(), static_cast<size_t>(workspace->element_count()));
  return status(rc, "lp_fwd");
}

// shard_stats [P, 3, T] f32 -> logp [T] f32, norm [2, T] f32
ffi::Error CombineImpl(cudaStream_t stream, ffi::Buffer<ffi::F32> shard_stats, ffi::ResultBuffer<ffi::F32> logp,
                       ffi::ResultBuffer<ffi::F32> norm) {
  const auto sd = shard_stats.dimensions();
  if (sd.size() != 3 || sd[1] != 3) return ffi::Error::InvalidArgument("lp_combine: stats must be [P, 3, T]");
  const int rc = lp_combine(stream, static_cast<const float*>(shard_stats.untyped_data()), static_cast<int>(sd[0]),
                            sd[2], static_cast<float*>(logp->untyped_data()), static_cast<float*>(norm->untyped_data()));
  return status(rc, "lp_combine");
}

// H, W, y, norm [2, T] f32, g [T] f32 -> dH [T, d] bf16, dW [Vs, d] f32, workspace u8
ffi::Error BwdImpl(cudaStream_t stream, ffi::Buffer<ffi::BF16> H, ffi::Buffer<ffi::BF16> W, ffi::Buffer<ffi::S32> y,
                   ffi::Buffer<ffi::F32> norm, ffi::Buffer<ffi::F32> g, ffi::ResultBuffer<ffi::BF16> dH,
                   ffi::ResultBuffer<ffi::F32> dW, ffi::ResultBuffer<ffi::U8> workspace, float softcap, int64_t v_off,
                   int64_t token_chunk) {
  const auto hd = H.dimensions();
  const auto wd = W.dimensions();
  if (hd.size() != 2 || wd.size() != 2) return ffi::Error::InvalidArgument("lp_bwd: H and W must be rank 2");
  const int rc =
      lp_bwd(stream, H.untyped_data(), hd[0], hd[1], hd[1], W.untyped_data(), wd[0], v_off,
             static_cast<const int32_t*>(y.untyped_data()), softcap, static_cast<const float*>(norm.untyped_data()),
             static_cast<const float*>(g.untyped_data()), dH->untyped_data(), hd[1], dW->untyped_data(), 0,
             token_chunk, workspace->untyped_data(), static_cast<size_t>(workspace->element_count()));
  return status(rc, "lp_bwd");
}

}  // namespace

XLA_FFI_DEFINE_HANDLER_SYMBOL(LpFwd, FwdImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::BF16>>()
                                  .Arg<ffi::Buffer<ffi::BF16>>()
                                  .Arg<ffi::Buffer<ffi::S32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::U8>>()
                                  .Attr<float>("softcap")
                                  .Attr<int64_t>("v_off"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(LpCombine, CombineImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>());

XLA_FFI_DEFINE_HANDLER_SYMBOL(LpBwd, BwdImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::BF16>>()
                                  .Arg<ffi::Buffer<ffi::BF16>>()
                                  .Arg<ffi::Buffer<ffi::S32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::BF16>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::U8>>()
                                  .Attr<float>("softcap")
                                  .Attr<int64_t>("v_off")
                                  .Attr<int64_t>("token_chunk"));

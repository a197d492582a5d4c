// XLA FFI handlers over libufp8 (include/ufp8.h): the binding through which the reference's JAX
// code calls this library as XLA custom calls (jax.ffi.register_ffi_target with these symbols,
// platform "CUDA"; jax.ffi.ffi_call from a custom_vjp that replaces the jnp.einsum of
// ueaj/model/einsum.py:243).  Compiled only against jaxlib's headers (xla/ffi/api/ffi.h):
// macrogpt_jax_b200/build.py builds lib/libufp8_xla.so when `jax` is importable and skips it
// otherwise.  Every buffer comes from XLA; the handlers allocate nothing and never synchronise.
//
// Return codes map to ffi errors: UFP8_ERR_INVALID / UFP8_ERR_ALIGN -> kInvalidArgument,
// UFP8_ERR_UNSUPPORTED -> kUnimplemented, UFP8_ERR_DEVICE -> kFailedPrecondition, anything
// else -> kInternal, each with ufp8_last_error()'s message.
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "ufp8.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

ffi::Error status(int rc) {
  if (rc == UFP8_OK) return ffi::Error::Success();
  ffi::ErrorCode code = ffi::ErrorCode::kInternal;
  if (rc == UFP8_ERR_INVALID || rc == UFP8_ERR_ALIGN) code = ffi::ErrorCode::kInvalidArgument;
  if (rc == UFP8_ERR_UNSUPPORTED) code = ffi::ErrorCode::kUnimplemented;
  if (rc == UFP8_ERR_DEVICE) code = ffi::ErrorCode::kFailedPrecondition;
  return ffi::Error(code, std::string("ufp8: ") + ufp8_last_error());
}

ufp8_stream_t st(cudaStream_t s) { return reinterpret_cast<ufp8_stream_t>(s); }

// x (bf16, any shape) -> q (fp8 of the same shape), amax (f32[1]), inv_scale (f32[1]).
// fmt: 0 = float8_e4m3fn (forward operands), 1 = float8_e5m2 (gradients).
ffi::Error AmaxQuantImpl(cudaStream_t s, ffi::AnyBuffer x, ffi::Result<ffi::AnyBuffer> q,
                         ffi::Result<ffi::Buffer<ffi::F32>> amax, ffi::Result<ffi::Buffer<ffi::F32>> inv, int32_t fmt) {
  return status(ufp8_amax_quant(x.untyped_data(), static_cast<int64_t>(x.element_count()), fmt, q->untyped_data(),
                                amax->typed_data(), inv->typed_data(), st(s)));
}

// The same without the amax output: the scratch is the library's static device array.
ffi::Error AmaxQuantNoallocImpl(cudaStream_t s, ffi::AnyBuffer x, ffi::Result<ffi::AnyBuffer> q,
                                ffi::Result<ffi::Buffer<ffi::F32>> inv, int32_t fmt) {
  return status(ufp8_amax_quant_noalloc(x.untyped_data(), static_cast<int64_t>(x.element_count()), fmt,
                                        q->untyped_data(), inv->typed_data(), st(s)));
}

// The GEMM view of an Einsum (EinsumMetadata, ueaj/model/einsum.py:67-147):
// D[g] = sum_kb A[g or kb] B[g or kb]^T * inv_a * inv_b, bf16 D [batch, M, N].
ffi::Error GemmImpl(cudaStream_t s, ffi::AnyBuffer a, ffi::Buffer<ffi::F32> inv_a, ffi::AnyBuffer b,
                    ffi::Buffer<ffi::F32> inv_b, ffi::Result<ffi::AnyBuffer> d, int64_t m, int64_t n, int64_t k,
                    int32_t a_fmt, int32_t a_major, int32_t a_slices, int32_t b_fmt, int32_t b_major,
                    int32_t b_slices, int32_t batch, int32_t k_batches) {
  ufp8_gemm_desc g = {};
  g.M = m;
  g.N = n;
  g.K = k;
  g.batch = batch;
  g.k_batches = k_batches;
  g.a.ptr = a.untyped_data();
  g.a.fmt = a_fmt;
  g.a.major = a_major;
  g.a.ld = a_major == UFP8_K_MAJOR ? k : m;
  g.a.batch_stride = m * k;
  g.a.batch_count = a_slices;
  g.a.inv_scale = inv_a.typed_data();
  g.b.ptr = b.untyped_data();
  g.b.fmt = b_fmt;
  g.b.major = b_major;
  g.b.ld = b_major == UFP8_K_MAJOR ? k : n;
  g.b.batch_stride = n * k;
  g.b.batch_count = b_slices;
  g.b.inv_scale = inv_b.typed_data();
  g.d = d->untyped_data();
  g.d_dtype = UFP8_OUT_BF16;
  g.epilogue = UFP8_EPI_STORE;
  g.ldd = n;
  g.d_batch_stride = m * n;
  return status(ufp8_gemm(&g, st(s)));
}

// GMLP gate/up projection with the fused gating (ueaj/model/mlp.py:78-86,102-107):
// x e4m3 [T, d], wf e4m3 [2, d, h] -> ug bf16 [2, T, h], h bf16 [T, h], amax_h f32[1].
ffi::Error GmlpF1Impl(cudaStream_t s, ffi::AnyBuffer x, ffi::Buffer<ffi::F32> inv_x, ffi::AnyBuffer wf,
                      ffi::Buffer<ffi::F32> inv_wf, ffi::Result<ffi::AnyBuffer> ug, ffi::Result<ffi::AnyBuffer> hid,
                      ffi::Result<ffi::Buffer<ffi::F32>> amax_h, int64_t t, int64_t dm, int64_t hd) {
  ufp8_gemm_desc g = {};
  g.M = t;
  g.N = hd;
  g.K = dm;
  g.batch = 1;
  g.k_batches = 1;
  g.a = {x.untyped_data(), UFP8_E4M3, UFP8_K_MAJOR, dm, 0, 1, 0, inv_x.typed_data()};
  g.b = {wf.untyped_data(), UFP8_E4M3, UFP8_MN_MAJOR, hd, dm * hd, 2, 0, inv_wf.typed_data()};
  g.d = ug->untyped_data();
  g.d_dtype = UFP8_OUT_BF16;
  g.epilogue = UFP8_EPI_SWIGLU;
  g.ldd = hd;
  g.d_batch_stride = t * hd;
  g.h = hid->untyped_data();
  g.ldh = hd;
  g.amax_out = amax_h->typed_data();
  return status(ufp8_gemm(&g, st(s)));
}

// dH = dY Wd^T fused with the gating backward: dy e5m2 [T, d], wd e4m3 [h, d], ug bf16 [2, T, h]
// -> dug bf16 [2, T, h], amax f32[1].
ffi::Error GmlpB2Impl(cudaStream_t s, ffi::AnyBuffer dy, ffi::Buffer<ffi::F32> inv_dy, ffi::AnyBuffer wd,
                      ffi::Buffer<ffi::F32> inv_wd, ffi::AnyBuffer ug, ffi::Result<ffi::AnyBuffer> dug,
                      ffi::Result<ffi::Buffer<ffi::F32>> amax, int64_t t, int64_t dm, int64_t hd) {
  ufp8_gemm_desc g = {};
  g.M = t;
  g.N = hd;
  g.K = dm;
  g.batch = 1;
  g.k_batches = 1;
  g.a = {dy.untyped_data(), UFP8_E5M2, UFP8_K_MAJOR, dm, 0, 1, 0, inv_dy.typed_data()};
  g.b = {wd.untyped_data(), UFP8_E4M3, UFP8_K_MAJOR, dm, 0, 1, 0, inv_wd.typed_data()};
  g.d = dug->untyped_data();
  g.d_dtype = UFP8_OUT_BF16;
  g.epilogue = UFP8_EPI_DSWIGLU;
  g.ldd = hd;
  g.d_batch_stride = t * hd;
  g.ug = ug.untyped_data();
  g.ldug = hd;
  g.ug_batch_stride = t * hd;
  g.amax_out = amax->typed_data();
  return status(ufp8_gemm(&g, st(s)));
}

// RMSNorm (ueaj/model/rmsnorm.py:68-84) fused with the e4m3 quantisation of its output:
// x bf16 [rows, d], scale bf16 [d] -> q e4m3 [rows, d], amax f32[1], inv f32[1], rstd f32[rows].
ffi::Error RmsnormQuantImpl(cudaStream_t s, ffi::AnyBuffer x, ffi::AnyBuffer scale, ffi::Result<ffi::AnyBuffer> q,
                            ffi::Result<ffi::Buffer<ffi::F32>> amax, ffi::Result<ffi::Buffer<ffi::F32>> inv,
                            ffi::Result<ffi::Buffer<ffi::F32>> rstd, int64_t rows, int64_t dm, int32_t centered,
                            float eps) {
  return status(ufp8_rmsnorm_quant(x.untyped_data(), rows, dm, dm, scale.untyped_data(),
                                   static_cast<int64_t>(scale.element_count()), centered, eps, UFP8_E4M3,
                                   q->untyped_data(), amax->typed_data(), inv->typed_data(), rstd->typed_data(),
                                   nullptr, 0, st(s)));
}

// Causal segment-masked GQA softmax attention (the flash_attention call of
// ueaj/model/soft_attn.py:186-196) with the default positions 0..n-1: q bf16 [b, n, h * i, d],
// k / v bf16 [b, n, h, d], segment ids s32 [b, n] (queries and keys alike) -> out bf16 like q,
// `saved` (P and lse, kept for the backward) and the scratch `workspace`; both byte sizes come from
// ufp8_attention_workspace for the same shape.
ufp8_attn_desc attn_desc(int64_t batch, int64_t seq, int64_t kv_heads, int64_t group, int64_t head_dim,
                         const int32_t* seg, float scale) {
  ufp8_attn_desc d = {};
  d.batch = batch;
  d.seq = seq;
  d.kv_heads = kv_heads;
  d.group = group;
  d.head_dim = head_dim;
  d.q_segment_ids = seg;
  d.kv_segment_ids = seg;
  d.scale = scale;
  return d;
}

ffi::Error AttentionForwardImpl(cudaStream_t s, ffi::AnyBuffer q, ffi::AnyBuffer k, ffi::AnyBuffer v,
                                ffi::Buffer<ffi::S32> seg, ffi::Result<ffi::AnyBuffer> out,
                                ffi::Result<ffi::AnyBuffer> saved, ffi::Result<ffi::AnyBuffer> workspace,
                                int64_t batch, int64_t seq, int64_t kv_heads, int64_t group, int64_t head_dim,
                                float scale) {
  const ufp8_attn_desc d = attn_desc(batch, seq, kv_heads, group, head_dim, seg.typed_data(), scale);
  return status(ufp8_attention_forward(&d, q.untyped_data(), k.untyped_data(), v.untyped_data(), out->untyped_data(),
                                       saved->untyped_data(), workspace->untyped_data(), st(s)));
}

// Its backward: dq, dk, dv (bf16, shaped like q, k, v) from dout at out and the forward's `saved`.
ffi::Error AttentionBackwardImpl(cudaStream_t s, ffi::AnyBuffer q, ffi::AnyBuffer k, ffi::AnyBuffer v,
                                 ffi::Buffer<ffi::S32> seg, ffi::AnyBuffer out, ffi::AnyBuffer dout,
                                 ffi::AnyBuffer saved, ffi::Result<ffi::AnyBuffer> dq, ffi::Result<ffi::AnyBuffer> dk,
                                 ffi::Result<ffi::AnyBuffer> dv, ffi::Result<ffi::AnyBuffer> workspace, int64_t batch,
                                 int64_t seq, int64_t kv_heads, int64_t group, int64_t head_dim, float scale) {
  const ufp8_attn_desc d = attn_desc(batch, seq, kv_heads, group, head_dim, seg.typed_data(), scale);
  return status(ufp8_attention_backward(&d, q.untyped_data(), k.untyped_data(), v.untyped_data(), out.untyped_data(),
                                        dout.untyped_data(), saved.untyped_data(), dq->untyped_data(),
                                        dk->untyped_data(), dv->untyped_data(), workspace->untyped_data(), st(s)));
}

}  // namespace

XLA_FFI_DEFINE_HANDLER_SYMBOL(Ufp8AmaxQuant, AmaxQuantImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Attr<int32_t>("fmt"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(Ufp8AmaxQuantNoalloc, AmaxQuantNoallocImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Attr<int32_t>("fmt"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(Ufp8Gemm, GemmImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Attr<int64_t>("m")
                                  .Attr<int64_t>("n")
                                  .Attr<int64_t>("k")
                                  .Attr<int32_t>("a_fmt")
                                  .Attr<int32_t>("a_major")
                                  .Attr<int32_t>("a_slices")
                                  .Attr<int32_t>("b_fmt")
                                  .Attr<int32_t>("b_major")
                                  .Attr<int32_t>("b_slices")
                                  .Attr<int32_t>("batch")
                                  .Attr<int32_t>("k_batches"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(Ufp8GmlpF1, GmlpF1Impl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Attr<int64_t>("tokens")
                                  .Attr<int64_t>("model_d")
                                  .Attr<int64_t>("hidden_d"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(Ufp8GmlpB2, GmlpB2Impl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Attr<int64_t>("tokens")
                                  .Attr<int64_t>("model_d")
                                  .Attr<int64_t>("hidden_d"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(Ufp8RmsnormQuant, RmsnormQuantImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Attr<int64_t>("rows")
                                  .Attr<int64_t>("model_d")
                                  .Attr<int32_t>("centered")
                                  .Attr<float>("eps"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(Ufp8AttentionForward, AttentionForwardImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::S32>>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Attr<int64_t>("batch")
                                  .Attr<int64_t>("seq")
                                  .Attr<int64_t>("kv_heads")
                                  .Attr<int64_t>("group")
                                  .Attr<int64_t>("head_dim")
                                  .Attr<float>("scale"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(Ufp8AttentionBackward, AttentionBackwardImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::S32>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Attr<int64_t>("batch")
                                  .Attr<int64_t>("seq")
                                  .Attr<int64_t>("kv_heads")
                                  .Attr<int64_t>("group")
                                  .Attr<int64_t>("head_dim")
                                  .Attr<float>("scale"));

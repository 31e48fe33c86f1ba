// XLA FFI handlers that expose libflexattn to JAX as CUDA custom calls.
//
// Build on a host with jaxlib (its FFI headers) and the built libflexattn.so:
//   g++ -std=c++17 -O2 -shared -fPIC flexattn_jax_ffi.cc \
//       -I"$(python -c 'import jax.ffi as f; print(f.include_dir())')" -I../../include \
//       -I/usr/local/cuda/include -L../pallas_flexattn -lflexattn -o libflexattn_jax.so
// and register from Python (see pallas_flexattn_jax.py):
//   jax.ffi.register_ffi_target("flexattn_fwd", jax.ffi.pycapsule(lib.FlexAttnFwd), platform="CUDA")
//
// Each handler maps XLA buffers (q/k/v/o in (B, H, T, D) row-major, block tables
// as int32 buffers) and attributes (mask/score parameters, scale, kernel choice)
// onto the plain C structs of include/flexattn.h and calls the C entry point on
// XLA's stream.  Layouts and semantics are those of flash_attention_fwd /
// flash_attention_bwd in the reference (src/pallas_flexattn/flash_attn.py:111-165,
// 410-461); the residuals (q, k, v, o, lse) are the reference's custom_vjp
// residuals (flash_attn.py:487).
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "flexattn.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

int32_t dtype_of(ffi::DataType t) {
  return t == ffi::DataType::BF16 ? FA_DTYPE_BF16 : (t == ffi::DataType::F32 ? FA_DTYPE_F32 : -1);
}

// Contiguous (B, H, T, D) buffer -> FaTensor.
FaTensor tensor_of(ffi::AnyBuffer buf) {
  auto d = buf.dimensions();
  FaTensor t;
  t.ptr = buf.untyped_data();
  t.stride_t = d[3];
  t.stride_h = d[2] * d[3];
  t.stride_b = d[1] * d[2] * d[3];
  return t;
}

ffi::Error status_of(int rc) {
  if (rc == FA_OK) return ffi::Error::Success();
  return ffi::Error(ffi::ErrorCode::kInternal, std::string("libflexattn: ") + fa_last_error());
}

struct Attrs {
  int32_t mask_flags, window_left, window_right, table_block, score_flags, block_size, kernel, num_stages;
  float softcap, scale;
};

void fill_common(const Attrs& at, ffi::AnyBuffer q, ffi::AnyBuffer k, ffi::Buffer<ffi::S32> doc,
                 ffi::Buffer<ffi::U8> tile_table, ffi::Buffer<ffi::F32> slopes, ffi::Buffer<ffi::F32> rel_bias,
                 ffi::Buffer<ffi::S32> kv_num, ffi::Buffer<ffi::S32> kv_idx, ffi::Buffer<ffi::S32> fkv_num,
                 ffi::Buffer<ffi::S32> fkv_idx, ffi::Buffer<ffi::S32> q_num, ffi::Buffer<ffi::S32> q_idx,
                 ffi::Buffer<ffi::S32> fq_num, ffi::Buffer<ffi::S32> fq_idx, int32_t* B, int32_t* H, int32_t* Hkv,
                 int32_t* Tq, int32_t* Tkv, int32_t* D, FaMaskSpec* m, FaScoreSpec* s, FaBlockTables* bt) {
  auto dq = q.dimensions(), dk = k.dimensions();
  *B = (int32_t)dq[0]; *H = (int32_t)dq[1]; *Tq = (int32_t)dq[2]; *D = (int32_t)dq[3];
  *Hkv = (int32_t)dk[1]; *Tkv = (int32_t)dk[2];
  *m = FaMaskSpec{};
  m->flags = at.mask_flags;
  m->window_left = at.window_left;
  m->window_right = at.window_right;
  if (at.mask_flags & FA_MASK_DOCUMENT) {
    m->doc_q = m->doc_kv = doc.typed_data();
    auto dd = doc.dimensions();
    m->doc_stride_b = (dd.size() == 2 && dd[0] > 1) ? dd[1] : 0;
  }
  if (at.mask_flags & FA_MASK_TILE_TABLE) {
    auto td = tile_table.dimensions();
    m->tile_table = tile_table.typed_data();
    m->table_rows = (int32_t)td[0];
    m->table_cols = (int32_t)td[1];
    m->table_block = at.table_block;
  }
  *s = FaScoreSpec{};
  s->flags = at.score_flags;
  s->softcap = at.softcap;
  if (at.score_flags & FA_SCORE_ALIBI) s->alibi_slopes = slopes.typed_data();
  if (at.score_flags & FA_SCORE_REL_BIAS) {
    auto bd = rel_bias.dimensions();
    s->rel_bias = rel_bias.typed_data();
    s->rel_bias_stride_h = bd[0] > 1 ? bd[1] : 0;
  }
  // tables: [num_b, 1, n] and [num_b, 1, n, cap]
  auto kd = kv_idx.dimensions(), qd = q_idx.dimensions();
  *bt = FaBlockTables{};
  bt->block_q = bt->block_kv = at.block_size;
  bt->nq = (int32_t)kd[kd.size() - 2];
  bt->nkv = (int32_t)qd[qd.size() - 2];
  bt->num_b = (int32_t)kd[0];
  bt->num_h = 1;
  bt->kv_num_blocks = kv_num.typed_data();
  bt->kv_indices = kv_idx.typed_data();
  bt->full_kv_num_blocks = fkv_num.typed_data();
  bt->full_kv_indices = fkv_idx.typed_data();
  bt->kv_cap = (int32_t)kd[kd.size() - 1];
  bt->q_num_blocks = q_num.typed_data();
  bt->q_indices = q_idx.typed_data();
  bt->full_q_num_blocks = fq_num.typed_data();
  bt->full_q_indices = fq_idx.typed_data();
  bt->q_cap = (int32_t)qd[qd.size() - 1];
}

#define FA_TABLE_ARGS                                                                                    \
  .Arg<ffi::Buffer<ffi::S32>>() /* doc ids */                                                            \
      .Arg<ffi::Buffer<ffi::U8>>() /* tile table */                                                      \
      .Arg<ffi::Buffer<ffi::F32>>() /* alibi slopes */                                                   \
      .Arg<ffi::Buffer<ffi::F32>>() /* relative bias */                                                  \
      .Arg<ffi::Buffer<ffi::S32>>()                                                                      \
      .Arg<ffi::Buffer<ffi::S32>>()                                                                      \
      .Arg<ffi::Buffer<ffi::S32>>()                                                                      \
      .Arg<ffi::Buffer<ffi::S32>>()                                                                      \
      .Arg<ffi::Buffer<ffi::S32>>()                                                                      \
      .Arg<ffi::Buffer<ffi::S32>>()                                                                      \
      .Arg<ffi::Buffer<ffi::S32>>()                                                                      \
      .Arg<ffi::Buffer<ffi::S32>>()

#define FA_ATTRS                                                                                         \
  .Attr<int32_t>("mask_flags")                                                                           \
      .Attr<int32_t>("window_left")                                                                      \
      .Attr<int32_t>("window_right")                                                                     \
      .Attr<int32_t>("table_block")                                                                      \
      .Attr<int32_t>("score_flags")                                                                      \
      .Attr<float>("softcap")                                                                            \
      .Attr<float>("scale")                                                                              \
      .Attr<int32_t>("block_size")                                                                       \
      .Attr<int32_t>("kernel")                                                                           \
      .Attr<int32_t>("num_stages")

ffi::Error FwdImpl(cudaStream_t stream, ffi::AnyBuffer q, ffi::AnyBuffer k, ffi::AnyBuffer v,
                   ffi::Buffer<ffi::S32> doc, ffi::Buffer<ffi::U8> table, ffi::Buffer<ffi::F32> slopes,
                   ffi::Buffer<ffi::F32> bias, ffi::Buffer<ffi::S32> kvn, ffi::Buffer<ffi::S32> kvi,
                   ffi::Buffer<ffi::S32> fkvn, ffi::Buffer<ffi::S32> fkvi, ffi::Buffer<ffi::S32> qn,
                   ffi::Buffer<ffi::S32> qi, ffi::Buffer<ffi::S32> fqn, ffi::Buffer<ffi::S32> fqi,
                   ffi::Result<ffi::AnyBuffer> o, ffi::Result<ffi::Buffer<ffi::F32>> lse, int32_t mask_flags,
                   int32_t window_left, int32_t window_right, int32_t table_block, int32_t score_flags,
                   float softcap, float scale, int32_t block_size, int32_t kernel, int32_t num_stages) {
  Attrs at{mask_flags, window_left, window_right, table_block, score_flags, block_size, kernel, num_stages,
           softcap, scale};
  FaFwdParams p{};
  p.dtype = dtype_of(q.element_type());
  fill_common(at, q, k, doc, table, slopes, bias, kvn, kvi, fkvn, fkvi, qn, qi, fqn, fqi, &p.B, &p.H, &p.H_kv,
              &p.Tq, &p.Tkv, &p.D, &p.mask, &p.score, &p.blocks);
  p.q = tensor_of(q);
  p.k = tensor_of(k);
  p.v = tensor_of(v);
  p.o = tensor_of(*o);
  p.lse = lse->typed_data();
  p.scale = scale;
  p.kernel = kernel;
  p.num_stages = num_stages;
  return status_of(fa_fwd(&p, reinterpret_cast<fa_stream_t>(stream)));
}

ffi::Error BwdImpl(cudaStream_t stream, ffi::AnyBuffer q, ffi::AnyBuffer k, ffi::AnyBuffer v, ffi::AnyBuffer o,
                   ffi::Buffer<ffi::F32> lse, ffi::AnyBuffer dout, ffi::Buffer<ffi::S32> doc,
                   ffi::Buffer<ffi::U8> table, ffi::Buffer<ffi::F32> slopes, ffi::Buffer<ffi::F32> bias,
                   ffi::Buffer<ffi::S32> kvn, ffi::Buffer<ffi::S32> kvi, ffi::Buffer<ffi::S32> fkvn,
                   ffi::Buffer<ffi::S32> fkvi, ffi::Buffer<ffi::S32> qn, ffi::Buffer<ffi::S32> qi,
                   ffi::Buffer<ffi::S32> fqn, ffi::Buffer<ffi::S32> fqi, ffi::Result<ffi::AnyBuffer> dq,
                   ffi::Result<ffi::AnyBuffer> dk, ffi::Result<ffi::AnyBuffer> dv,
                   ffi::Result<ffi::Buffer<ffi::U8>> workspace, int32_t mask_flags, int32_t window_left,
                   int32_t window_right, int32_t table_block, int32_t score_flags, float softcap, float scale,
                   int32_t block_size, int32_t kernel, int32_t num_stages) {
  Attrs at{mask_flags, window_left, window_right, table_block, score_flags, block_size, kernel, num_stages,
           softcap, scale};
  FaBwdParams p{};
  p.dtype = dtype_of(q.element_type());
  fill_common(at, q, k, doc, table, slopes, bias, kvn, kvi, fkvn, fkvi, qn, qi, fqn, fqi, &p.B, &p.H, &p.H_kv,
              &p.Tq, &p.Tkv, &p.D, &p.mask, &p.score, &p.blocks);
  p.q = tensor_of(q);
  p.k = tensor_of(k);
  p.v = tensor_of(v);
  p.o = tensor_of(o);
  p.dout = tensor_of(dout);
  p.dq = tensor_of(*dq);
  p.dk = tensor_of(*dk);
  p.dv = tensor_of(*dv);
  p.lse = lse.typed_data();
  p.scale = scale;
  p.kernel = kernel;
  p.num_stages = num_stages;
  return status_of(fa_bwd(&p, workspace->untyped_data(), workspace->size_bytes(),
                          reinterpret_cast<fa_stream_t>(stream)));
}

// create_block_mask on the GPU (reference block_mask.py:54-129): tile classes and the
// row / column tables for a registry mask.
ffi::Error BlockMaskImpl(cudaStream_t stream, ffi::Buffer<ffi::S32> doc, ffi::Buffer<ffi::U8> table,
                         ffi::Result<ffi::Buffer<ffi::U8>> cls, ffi::Result<ffi::Buffer<ffi::S32>> kvn,
                         ffi::Result<ffi::Buffer<ffi::S32>> kvi, ffi::Result<ffi::Buffer<ffi::S32>> fkvn,
                         ffi::Result<ffi::Buffer<ffi::S32>> fkvi, ffi::Result<ffi::Buffer<ffi::S32>> qn,
                         ffi::Result<ffi::Buffer<ffi::S32>> qi, ffi::Result<ffi::Buffer<ffi::S32>> fqn,
                         ffi::Result<ffi::Buffer<ffi::S32>> fqi, int32_t mask_flags, int32_t window_left,
                         int32_t window_right, int32_t table_block, int32_t B, int32_t Tq, int32_t Tkv,
                         int32_t block_size, int32_t mode) {
  FaMaskSpec m{};
  m.flags = mask_flags;
  m.window_left = window_left;
  m.window_right = window_right;
  if (mask_flags & FA_MASK_DOCUMENT) {
    auto dd = doc.dimensions();
    m.doc_q = m.doc_kv = doc.typed_data();
    m.doc_stride_b = (dd.size() == 2 && dd[0] > 1) ? dd[1] : 0;
  }
  if (mask_flags & FA_MASK_TILE_TABLE) {
    auto td = table.dimensions();
    m.tile_table = table.typed_data();
    m.table_rows = (int32_t)td[0];
    m.table_cols = (int32_t)td[1];
    m.table_block = table_block;
  }
  auto cd = cls->dimensions();
  FaBlockMaskOut out{};
  out.num_b = (int32_t)cd[0];
  out.nq = (int32_t)cd[1];
  out.nkv = (int32_t)cd[2];
  out.tile_class = cls->typed_data();
  out.kv_num_blocks = kvn->typed_data();
  out.kv_indices = kvi->typed_data();
  out.full_kv_num_blocks = fkvn->typed_data();
  out.full_kv_indices = fkvi->typed_data();
  out.q_num_blocks = qn->typed_data();
  out.q_indices = qi->typed_data();
  out.full_q_num_blocks = fqn->typed_data();
  out.full_q_indices = fqi->typed_data();
  return status_of(fa_create_block_mask(&m, B, Tq, Tkv, block_size, block_size, mode, &out,
                                        reinterpret_cast<fa_stream_t>(stream)));
}

}  // namespace

XLA_FFI_DEFINE_HANDLER_SYMBOL(FlexAttnBlockMask, BlockMaskImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::S32>>()
                                  .Arg<ffi::Buffer<ffi::U8>>()
                                  .Ret<ffi::Buffer<ffi::U8>>()
                                  .Ret<ffi::Buffer<ffi::S32>>()
                                  .Ret<ffi::Buffer<ffi::S32>>()
                                  .Ret<ffi::Buffer<ffi::S32>>()
                                  .Ret<ffi::Buffer<ffi::S32>>()
                                  .Ret<ffi::Buffer<ffi::S32>>()
                                  .Ret<ffi::Buffer<ffi::S32>>()
                                  .Ret<ffi::Buffer<ffi::S32>>()
                                  .Ret<ffi::Buffer<ffi::S32>>()
                                  .Attr<int32_t>("mask_flags")
                                  .Attr<int32_t>("window_left")
                                  .Attr<int32_t>("window_right")
                                  .Attr<int32_t>("table_block")
                                  .Attr<int32_t>("B")
                                  .Attr<int32_t>("Tq")
                                  .Attr<int32_t>("Tkv")
                                  .Attr<int32_t>("block_size")
                                  .Attr<int32_t>("mode"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(FlexAttnFwd, FwdImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>() FA_TABLE_ARGS.Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::F32>>() FA_ATTRS);

XLA_FFI_DEFINE_HANDLER_SYMBOL(FlexAttnBwd, BwdImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::AnyBuffer>() FA_TABLE_ARGS.Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::U8>>() FA_ATTRS);

// torch.ops.kvr.*: the per-call decode path as C++ PyTorch operators.
//
// The draft model's attention calls decode attention once per layer and
// token (kv_reduce/experiments/packed_review.py:68-79 hooks it into the
// model), so the host cost of that call is paid ~28 times per token.  These
// operators do the reference's argument checks
// (kv_reduce/triton_packed_kv_attention.py:293-314, same order and messages,
// raised as ValueError), derive the (b, h) slab strides and device pointers,
// allocate the output and call the extern "C" launchers of libkvr.so, all
// in C++:
//
//   kvr::decode_attention  <- packed_kv_decode_attention (:284-389)
//   kvr::decode_step       <- PackedLayer.append + the attention call on a
//                             streaming layer (packed_review.py:23-31, :78):
//                             one launch that appends the token and decodes
//                             with lengths kept in device memory
//   kvr::lse_merge         <- the LSE merge of per-shard partials (:251-281)
//
// No CUDA code lives here: the kernels are libkvr.so's.  Outputs come from
// the caching allocator; the split workspace and merge counters are cached
// per (device, stream) and grown on demand (a completed launch leaves the
// counters at zero, so stream-ordered launches share them).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <array>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <utility>

#include "../../include/kvr.h"

namespace {

void raise_status(const char* fn, int st) {
  if (st == KVR_OK) return;
  const std::string text = kvr_status_string(st);
  if (st == KVR_ERR_INVALID_ARGUMENT || st == KVR_ERR_UNSUPPORTED || st == KVR_ERR_MISALIGNED)
    TORCH_CHECK_VALUE(false, fn, " failed: ", text, " (status ", st, ")");
  TORCH_CHECK(false, fn, " failed: ", text, " (status ", st, ")", st == KVR_ERR_CUDA ? ": " : "",
              st == KVR_ERR_CUDA ? kvr_last_error() : "");
}

// Stride between consecutive (b, h) slabs, in elements: `compact` for a
// contiguous tensor (the reference's layout), else dim 1's stride of a
// [B, H, ...] view into a capacity buffer with contiguous trailing dims.
int64_t bh_stride(const at::Tensor& t, int64_t compact, const char* what) {
  if (t.dim() <= 1 || t.is_contiguous()) return compact;
  TORCH_CHECK_VALUE(t.dim() >= 3 && t.stride(0) == t.size(1) * t.stride(1), what, ": unsupported strides ",
                    t.strides(), ".");
  int64_t expect = 1;
  for (int64_t d = t.dim() - 1; d >= 2; --d) {
    TORCH_CHECK_VALUE(t.size(d) == 1 || t.stride(d) == expect, what, ": inner dimensions must be contiguous.");
    expect *= t.size(d);
  }
  return t.stride(1);
}

const void* ptr_or_null(const std::optional<at::Tensor>& t) {
  return (t.has_value() && t->defined() && t->numel() > 0) ? t->data_ptr() : nullptr;
}

void check_on(const std::optional<at::Tensor>& t, const at::Device& dev) {
  if (t.has_value() && t->defined())
    TORCH_CHECK_VALUE(t->is_cuda() && t->device() == dev, "Packed K/V tensors must be on the query's CUDA device.");
}

struct Scratch {
  at::Tensor workspace, counters;
};
std::mutex g_mu;
std::map<std::pair<int, uintptr_t>, Scratch> g_scratch;

// Plans per geometry (the library memoises too; this skips the call).
struct PlanKey {
  std::array<int64_t, 12> v;
  bool operator<(const PlanKey& o) const { return v < o.v; }
};
std::map<PlanKey, std::array<int64_t, 3>> g_plans;

void attach_scratch(kvr_decode_args& a, const at::Device& dev, cudaStream_t stream) {
  PlanKey key{{a.batch, a.q_heads, a.kv_heads, a.head_dim, a.seq_len, a.prefix_len, a.group_size, a.key_bits,
               a.value_bits, a.split_tokens, a.n_layers, dev.index()}};
  std::array<int64_t, 3> plan;
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_plans.find(key);
  if (it == g_plans.end()) {
    int ns = 0;
    size_t ws = 0, cnt = 0;
    raise_status("kvr_decode_plan", kvr_decode_plan(&a, &ns, &ws, &cnt));
    plan = {ns, (int64_t)ws, (int64_t)cnt};
    g_plans.emplace(key, plan);
  } else {
    plan = it->second;
  }
  Scratch& s = g_scratch[{dev.index(), reinterpret_cast<uintptr_t>(stream)}];
  if (!s.workspace.defined() || s.workspace.numel() < plan[1])
    s.workspace = at::empty({std::max<int64_t>(plan[1], 1 << 16)}, at::TensorOptions().dtype(at::kByte).device(dev));
  if (!s.counters.defined() || s.counters.numel() < plan[2])
    s.counters = at::zeros({std::max<int64_t>(plan[2], 1024)}, at::TensorOptions().dtype(at::kInt).device(dev));
  a.workspace = s.workspace.data_ptr();
  a.workspace_bytes = (size_t)s.workspace.numel();
  a.counters = s.counters.data_ptr<int>();
}

constexpr int64_t kLayoutKeysOk = 1, kLayoutValuesOk = 2;

// shapes (optional) = the packed components' logical shapes
// [kB, kHKV, kS, kD, vB, vHKV, vS, vD]; without it the cache is taken to be
// [query batch, value_scale.size(1), seq_len, query head_dim].
// layouts = kLayoutKeysOk | kLayoutValuesOk when the components' layouts are
// per_channel_grouped_affine (keys) and per_token_affine (values).
at::Tensor decode_attention(const at::Tensor& query, const at::Tensor& key_payload,
                            const std::optional<at::Tensor>& key_scale, const std::optional<at::Tensor>& key_offset,
                            const std::optional<at::Tensor>& key_residual, const at::Tensor& value_payload,
                            const std::optional<at::Tensor>& value_scale,
                            const std::optional<at::Tensor>& value_offset, int64_t seq_len, int64_t kb, int64_t vb,
                            int64_t G, int64_t P, int64_t split, int64_t block, bool out_fp32,
                            at::OptionalIntArrayRef shapes, int64_t layouts,
                            const std::optional<at::Tensor>& key_scale_pairs) {
  // the reference's preconditions, in its order (:293-314)
  TORCH_CHECK_VALUE(query.is_cuda(), "Packed attention requires a CUDA query tensor.");
  TORCH_CHECK_VALUE(query.dim() == 4 && query.size(2) == 1, "query must have shape [batch, query_heads, 1, head_dim].");
  TORCH_CHECK_VALUE(layouts & kLayoutKeysOk, "keys must use the grouped per-channel affine layout.");
  TORCH_CHECK_VALUE(layouts & kLayoutValuesOk, "values must use the per-token affine layout.");
  auto bits_ok = [](int64_t b) { return b == 2 || b == 4 || b == 8; };
  TORCH_CHECK_VALUE(bits_ok(kb) && bits_ok(vb), "The fused kernel supports only 2-, 4- and 8-bit K/V payloads.");
  int64_t B, HKV, S, D;
  if (shapes.has_value()) {
    const at::IntArrayRef sh = *shapes;
    TORCH_CHECK_VALUE(sh.size() == 8, "shapes must hold the key and value shapes (8 integers).");
    TORCH_CHECK_VALUE(sh[0] == sh[4] && sh[1] == sh[5] && sh[2] == sh[6] && sh[3] == sh[7],
                      "Packed key and value shapes must match.");
    B = sh[0], HKV = sh[1], S = sh[2], D = sh[3];
  } else {
    TORCH_CHECK_VALUE(value_scale.has_value() && value_scale->dim() >= 2, "value scale must be [B, H, S, 1].");
    B = query.size(0), HKV = value_scale->size(1), S = seq_len, D = query.size(3);
  }
  TORCH_CHECK_VALUE(query.size(0) == B, "Query and cache batch dimensions must match.");
  TORCH_CHECK_VALUE(query.size(3) == D, "Query and cache head dimensions must match.");
  TORCH_CHECK_VALUE(HKV > 0 && query.size(1) % HKV == 0, "Query heads must be divisible by KV heads.");
  TORCH_CHECK_VALUE(P > 0, "The fused kernel requires a non-empty quantized key prefix.");
  TORCH_CHECK_VALUE(block == 16 || block == 32 || block == 64, "block_tokens must be one of 16, 32, or 64.");
  // geometry the kernel covers
  TORCH_CHECK_VALUE(D == 64 || D == 128, "head_dim must be one of [64, 128].");
  TORCH_CHECK_VALUE(!(D == 64 && vb == 2), "2-bit values need head_dim 128.");
  TORCH_CHECK_VALUE(query.size(1) / HKV <= 8, "At most 8 query heads per KV head are supported.");
  TORCH_CHECK_VALUE(G > 0 && G % 16 == 0, "group_size must be a multiple of 16 for the fused kernel.");
  TORCH_CHECK_VALUE(query.scalar_type() == at::kBFloat16, "query must be bf16.");
  TORCH_CHECK_VALUE(P <= S && P % G == 0, "prefix_len must be a multiple of group_size and at most seq_len.");
  const std::pair<const std::optional<at::Tensor>*, const char*> metas[] = {
      {&key_scale, "key scale"}, {&key_offset, "key offset"}, {&value_scale, "value scale"},
      {&value_offset, "value offset"}};
  for (const auto& m : metas)
    TORCH_CHECK_VALUE(m.first->has_value() && (*m.first)->defined() && (*m.first)->scalar_type() == at::kBFloat16,
                      m.second, " must be bf16.");
  const at::Device dev = query.device();
  TORCH_CHECK_VALUE(key_payload.is_cuda() && key_payload.device() == dev && value_payload.is_cuda() &&
                        value_payload.device() == dev,
                    "Packed K/V tensors must be on the query's CUDA device.");
  check_on(key_scale, dev);
  check_on(key_offset, dev);
  check_on(key_residual, dev);
  check_on(value_scale, dev);
  check_on(value_offset, dev);
  check_on(key_scale_pairs, dev);
  // the fp16 scale pairs are used only when laid out like the bf16 scales
  const void* pairs = nullptr;
  if (key_scale_pairs.has_value() && key_scale_pairs->defined() && key_scale_pairs->numel() > 0 &&
      key_scale_pairs->element_size() == 2 && key_scale_pairs->sizes() == key_scale->sizes() &&
      key_scale_pairs->strides() == key_scale->strides())
    pairs = key_scale_pairs->data_ptr();

  kvr_decode_args a;
  std::memset(&a, 0, sizeof(a));
  a.key_payload_bh_stride = bh_stride(key_payload, P * D * kb / 8, "key payload");
  a.key_meta_bh_stride = bh_stride(*key_scale, (P / G) * D, "key scale");
  TORCH_CHECK_VALUE(bh_stride(*key_offset, (P / G) * D, "key offset") == a.key_meta_bh_stride,
                    "key scale and offset must share strides.");
  if (S > P) {
    TORCH_CHECK_VALUE(key_residual.has_value() && key_residual->defined() &&
                          key_residual->scalar_type() == at::kBFloat16,
                      "key residual must be bf16.");
    a.key_residual_bh_stride = bh_stride(*key_residual, (S - P) * D, "key residual");
  }
  a.value_payload_bh_stride = bh_stride(value_payload, S * D * vb / 8, "value payload");
  a.value_meta_bh_stride = bh_stride(*value_scale, S, "value scale");
  TORCH_CHECK_VALUE(bh_stride(*value_offset, S, "value offset") == a.value_meta_bh_stride,
                    "value scale and offset must share strides.");

  c10::cuda::CUDAGuard guard(dev);
  const at::Tensor q = query.contiguous();
  at::Tensor out = out_fp32 ? at::empty(q.sizes(), q.options().dtype(at::kFloat)) : at::empty_like(q);
  kvr_layer_ptrs L;
  L.key_payload = static_cast<const uint8_t*>(ptr_or_null(key_payload));
  L.key_scale = static_cast<const uint16_t*>(ptr_or_null(key_scale));
  L.key_offset = static_cast<const uint16_t*>(ptr_or_null(key_offset));
  L.key_residual = static_cast<const uint16_t*>(ptr_or_null(key_residual));
  L.value_payload = static_cast<const uint8_t*>(ptr_or_null(value_payload));
  L.value_scale = static_cast<const uint16_t*>(ptr_or_null(value_scale));
  L.value_offset = static_cast<const uint16_t*>(ptr_or_null(value_offset));
  L.query = static_cast<const uint16_t*>(q.data_ptr());
  L.out = out.data_ptr();
  L.key_scale_pairs = static_cast<const uint16_t*>(pairs);
  a.layers = &L;
  a.n_layers = 1;
  a.batch = (int)B;
  a.q_heads = (int)q.size(1);
  a.kv_heads = (int)HKV;
  a.head_dim = (int)D;
  a.seq_len = (int)S;
  a.prefix_len = (int)P;
  a.group_size = (int)G;
  a.key_bits = (int)kb;
  a.value_bits = (int)vb;
  a.out_dtype = out_fp32 ? 1 : 0;
  // a positive split is rounded up to block_tokens (then to 32 by the library)
  a.split_tokens = split > 0 ? (int)((split + block - 1) / block * block) : 0;
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev.index()).stream();
  attach_scratch(a, dev, stream);
  raise_status("kvr_decode_attention", kvr_decode_attention(&a, stream));
  return out;
}

// One new token per (b, kv head) appended to a streaming layer's capacity
// buffers and attended to in the same launch (kvr_decode_step); the lengths
// live in `lengths` (int32[4] on the device) and advance on the device.
// geom = [capacity, prefix_capacity, residual_capacity, key_bits, value_bits,
//         group_size, split_tokens]
//
// Every argument check runs in check_step, before anything is allocated:
// decode_step raises its ValueError with no output tensor alive.
void check_step(const at::Tensor& query, const at::Tensor& k_new, const at::Tensor& v_new,
                const at::Tensor& key_payload, const at::Tensor& key_scale, const at::Tensor& key_offset,
                const at::Tensor& key_residual, const at::Tensor& value_payload, const at::Tensor& value_scale,
                const at::Tensor& value_offset, const at::Tensor& lengths, at::IntArrayRef geom,
                const std::optional<at::Tensor>& key_scale_pairs) {
  TORCH_CHECK_VALUE(geom.size() == 7, "kvr::decode_step: geom must hold 7 integers.");
  TORCH_CHECK_VALUE(query.is_cuda() && query.dim() == 4 && query.size(2) == 1 &&
                        query.scalar_type() == at::kBFloat16,
                    "query must be a bf16 CUDA tensor [batch, q_heads, 1, head_dim].");
  TORCH_CHECK_VALUE(value_payload.dim() >= 3, "value payload must be [batch, kv_heads, capacity, ...].");
  const int64_t B = value_payload.size(0), HKV = value_payload.size(1), D = query.size(3);
  TORCH_CHECK_VALUE(query.size(0) == B && query.size(1) % HKV == 0, "query must be bf16 [", B, ", q_heads, 1, ", D,
                    "] with q_heads a multiple of ", HKV, ".");
  TORCH_CHECK_VALUE(k_new.scalar_type() == at::kBFloat16 && v_new.scalar_type() == at::kBFloat16 &&
                        k_new.sizes() == v_new.sizes() && k_new.dim() == 4 && k_new.size(0) == B &&
                        k_new.size(1) == HKV && k_new.size(2) == 1 && k_new.size(3) == D,
                    "k/v must be bf16 [", B, ", ", HKV, ", 1, ", D, "].");
  const at::Device dev = query.device();
  const at::Tensor* tensors[] = {&k_new,   &v_new,         &key_payload, &key_scale,    &key_offset,
                                 &key_residual, &value_payload, &value_scale, &value_offset, &lengths};
  for (const at::Tensor* t : tensors)
    TORCH_CHECK_VALUE(t->is_cuda() && t->device() == dev, "All tensors must be on the query's CUDA device.");
  TORCH_CHECK_VALUE(lengths.scalar_type() == at::kInt && lengths.numel() >= 4 && lengths.is_contiguous(),
                    "lengths must be a contiguous int32[4] device tensor.");
  if (key_scale_pairs.has_value() && key_scale_pairs->defined())
    TORCH_CHECK_VALUE(key_scale_pairs->is_cuda() && key_scale_pairs->device() == dev &&
                          key_scale_pairs->element_size() == 2 && key_scale_pairs->sizes() == key_scale.sizes() &&
                          key_scale_pairs->strides() == key_scale.strides(),
                      "key_scale_pairs must be laid out like key_scale on the query's device.");
}

at::Tensor& decode_step_out(const at::Tensor& query, const at::Tensor& k_new, const at::Tensor& v_new,
                            const at::Tensor& key_payload, const at::Tensor& key_scale, const at::Tensor& key_offset,
                            const at::Tensor& key_residual, const at::Tensor& value_payload,
                            const at::Tensor& value_scale, const at::Tensor& value_offset, const at::Tensor& lengths,
                            at::IntArrayRef geom, const std::optional<at::Tensor>& key_scale_pairs,
                            at::Tensor& out) {
  check_step(query, k_new, v_new, key_payload, key_scale, key_offset, key_residual, value_payload, value_scale,
             value_offset, lengths, geom, key_scale_pairs);
  TORCH_CHECK_VALUE(out.sizes() == query.sizes() && out.scalar_type() == at::kBFloat16 && out.is_contiguous() &&
                        out.device() == query.device(),
                    "out must be a contiguous bf16 tensor like the query.");
  const int64_t cap = geom[0], cap_prefix = geom[1], cap_res = geom[2], kb = geom[3], vb = geom[4], G = geom[5],
                split = geom[6];
  const int64_t B = value_payload.size(0), HKV = value_payload.size(1), D = query.size(3);
  const at::Device dev = query.device();
  c10::cuda::CUDAGuard guard(dev);
  const at::Tensor q = query.contiguous(), k = k_new.contiguous(), v = v_new.contiguous();
  kvr_layer_ptrs L;
  L.key_payload = static_cast<const uint8_t*>(key_payload.data_ptr());
  L.key_scale = static_cast<const uint16_t*>(key_scale.data_ptr());
  L.key_offset = static_cast<const uint16_t*>(key_offset.data_ptr());
  L.key_residual = static_cast<const uint16_t*>(key_residual.data_ptr());
  L.value_payload = static_cast<const uint8_t*>(value_payload.data_ptr());
  L.value_scale = static_cast<const uint16_t*>(value_scale.data_ptr());
  L.value_offset = static_cast<const uint16_t*>(value_offset.data_ptr());
  L.query = static_cast<const uint16_t*>(q.data_ptr());
  L.out = out.data_ptr();
  L.key_scale_pairs = (key_scale_pairs.has_value() && key_scale_pairs->defined() && key_scale_pairs->numel() > 0)
                          ? static_cast<const uint16_t*>(key_scale_pairs->data_ptr())
                          : nullptr;
  kvr_decode_args a;
  std::memset(&a, 0, sizeof(a));
  a.layers = &L;
  a.n_layers = 1;
  a.batch = (int)B;
  a.q_heads = (int)q.size(1);
  a.kv_heads = (int)HKV;
  a.head_dim = (int)D;
  a.seq_len = (int)cap;
  a.prefix_len = (int)cap_prefix;
  a.group_size = (int)G;
  a.key_bits = (int)kb;
  a.value_bits = (int)vb;
  a.key_payload_bh_stride = key_payload.stride(1);
  a.key_meta_bh_stride = key_scale.stride(1);
  a.key_residual_bh_stride = key_residual.stride(1);
  a.value_payload_bh_stride = value_payload.stride(1);
  a.value_meta_bh_stride = value_scale.stride(1);
  a.split_tokens = (int)split;
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev.index()).stream();
  attach_scratch(a, dev, stream);
  raise_status("kvr_decode_step",
               kvr_decode_step(&a, static_cast<const uint16_t*>(k.data_ptr()),
                               static_cast<const uint16_t*>(v.data_ptr()), lengths.data_ptr<int>(), (int)cap_res,
                               stream));
  return out;
}

at::Tensor decode_step(const at::Tensor& query, const at::Tensor& k_new, const at::Tensor& v_new,
                       const at::Tensor& key_payload, const at::Tensor& key_scale, const at::Tensor& key_offset,
                       const at::Tensor& key_residual, const at::Tensor& value_payload, const at::Tensor& value_scale,
                       const at::Tensor& value_offset, const at::Tensor& lengths, at::IntArrayRef geom,
                       const std::optional<at::Tensor>& key_scale_pairs) {
  check_step(query, k_new, v_new, key_payload, key_scale, key_offset, key_residual, value_payload, value_scale,
             value_offset, lengths, geom, key_scale_pairs);
  at::Tensor out = at::empty(query.sizes(), query.options().memory_format(at::MemoryFormat::Contiguous));
  decode_step_out(query, k_new, v_new, key_payload, key_scale, key_offset, key_residual, value_payload, value_scale,
                  value_offset, lengths, geom, key_scale_pairs, out);
  return out;
}

at::Tensor lse_merge(const at::Tensor& part_ml, const at::Tensor& part_o) {
  TORCH_CHECK_VALUE(part_ml.dim() == 3 && part_ml.size(2) == 2 && part_o.dim() == 3,
                    "part_ml must be [n_parts, rows, 2] and part_o [n_parts, rows, D].");
  TORCH_CHECK_VALUE(part_ml.size(0) == part_o.size(0) && part_ml.size(1) == part_o.size(1),
                    "part_ml and part_o disagree on [n_parts, rows].");
  TORCH_CHECK_VALUE(part_ml.is_cuda() && part_o.is_cuda() && part_ml.device() == part_o.device(),
                    "kv_reduce_b200 operates on CUDA tensors only (no CPU fallback).");
  c10::cuda::CUDAGuard guard(part_ml.device());
  const at::Tensor ml = part_ml.to(at::kFloat).contiguous(), o = part_o.to(at::kFloat).contiguous();
  at::Tensor out = at::empty({o.size(1), o.size(2)}, o.options().dtype(at::kBFloat16));
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(part_ml.device().index()).stream();
  raise_status("kvr_lse_merge", kvr_lse_merge(ml.data_ptr<float>(), o.data_ptr<float>(), (int)o.size(0),
                                              (int)o.size(1), (int)o.size(2),
                                              static_cast<uint16_t*>(out.data_ptr()), stream));
  return out;
}

}  // namespace

TORCH_LIBRARY(kvr, m) {
  m.def("decode_attention(Tensor query, Tensor key_payload, Tensor? key_scale, Tensor? key_offset, "
        "Tensor? key_residual, Tensor value_payload, Tensor? value_scale, Tensor? value_offset, int seq_len, "
        "int key_bits, int value_bits, int group_size, int prefix_len, int split_tokens=0, int block_tokens=32, "
        "bool out_fp32=False, int[]? shapes=None, int layouts=3, Tensor? key_scale_pairs=None) -> Tensor");
  m.def("decode_step(Tensor query, Tensor k_new, Tensor v_new, Tensor key_payload, Tensor key_scale, "
        "Tensor key_offset, Tensor(a!) key_residual, Tensor(b!) value_payload, Tensor(c!) value_scale, "
        "Tensor(d!) value_offset, Tensor(e!) lengths, int[] geom, Tensor? key_scale_pairs=None) -> Tensor");
  m.def("decode_step.out(Tensor query, Tensor k_new, Tensor v_new, Tensor key_payload, Tensor key_scale, "
        "Tensor key_offset, Tensor(a!) key_residual, Tensor(b!) value_payload, Tensor(c!) value_scale, "
        "Tensor(d!) value_offset, Tensor(e!) lengths, int[] geom, Tensor? key_scale_pairs=None, *, "
        "Tensor(f!) out) -> Tensor(f!)");
  m.def("lse_merge(Tensor part_ml, Tensor part_o) -> Tensor");
}

TORCH_LIBRARY_IMPL(kvr, CUDA, m) {
  m.impl("decode_attention", &decode_attention);
  m.impl("decode_step", &decode_step);
  m.impl("decode_step.out", &decode_step_out);
  m.impl("lse_merge", &lse_merge);
}

// Host tensors reach the same functions, whose first check raises the
// reference's "requires a CUDA query" ValueError: there is no CPU path.
TORCH_LIBRARY_IMPL(kvr, CPU, m) {
  m.impl("decode_attention", &decode_attention);
  m.impl("decode_step", &decode_step);
  m.impl("decode_step.out", &decode_step_out);
  m.impl("lse_merge", &lse_merge);
}

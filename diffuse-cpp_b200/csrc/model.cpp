// model.cpp — whole-model upload from GGUF: one dmoe_layer per MoE block, bound once.
//
// Reference: diffuse_model_load_impl (src/diffuse-model.cpp:67-224): hyper-parameters through
// get_u32_multi / get_f32_multi (prefixes diffuse, qwen2, llama; :21-45, :141-158), the model
// type (:93-113), the MoE tensors of each block il >= first_k_dense (:184-196). The reference
// keeps the tensors in host memory and offloads nothing (src/diffuse-backend.h:104-118); here
// each MoE layer is copied to the device by dmoe_create as soon as its tensors are located, and
// the file mapping is released when the load returns.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "diffuse_moe.h"
#include "dmoe_internal.h"
#include "gguf.h"

using namespace dmoe;

struct dmoe_model {
  dmoe_model_info info{};
  std::vector<dmoe_layer*> layers;  // n_layer entries; nullptr for the dense blocks
};

namespace {

dmoe_status mfail(dmoe_status st, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  set_last_error(buf);
  return st;
}

const char* const kPrefixes[] = {"diffuse", "qwen2", "llama"};

// get_u32_multi: the first "<prefix>.<suffix>" present; the reference reads it as u32
// (gguf_get_val_u32 asserts the type), so another type is an error here
dmoe_status get_u32(const GgufFile& f, const char* suffix, bool required, uint32_t dflt, uint32_t& v) {
  for (const char* p : kPrefixes) {
    const std::string key = std::string(p) + "." + suffix;
    if (const GgufValue* kv = f.find(key)) {
      if (kv->type != GGUF_U32) return mfail(DMOE_ERR_INVALID_ARG, "GGUF key %s is not a u32", key.c_str());
      v = (uint32_t)kv->u;
      return DMOE_OK;
    }
  }
  if (required) return mfail(DMOE_ERR_INVALID_ARG, "missing GGUF key *.%s", suffix);
  v = dflt;
  return DMOE_OK;
}

dmoe_status get_f32(const GgufFile& f, const char* suffix, float dflt, float& v) {
  for (const char* p : kPrefixes) {
    const std::string key = std::string(p) + "." + suffix;
    if (const GgufValue* kv = f.find(key)) {
      if (kv->type != GGUF_F32) return mfail(DMOE_ERR_INVALID_ARG, "GGUF key %s is not an f32", key.c_str());
      v = (float)kv->f;
      return DMOE_OK;
    }
  }
  v = dflt;
  return DMOE_OK;
}

// the reference's model type: diffuse.model_type, else by architecture (:93-103, :47-54)
std::string model_type(const GgufFile& f) {
  if (const GgufValue* t = f.find("diffuse.model_type"); t && t->type == GGUF_STRING) return t->s;
  std::string arch = "unknown";
  if (const GgufValue* a = f.find("general.architecture"); a && a->type == GGUF_STRING) arch = a->s;
  else if (f.find("diffuse.block_count")) arch = "diffuse";
  else if (f.find("qwen2.block_count")) arch = "qwen2";
  else if (f.find("llama.block_count")) arch = "llama";
  if (arch == "qwen2") return "dream";
  if (arch == "llama") return "llada";
  return "llada2_moe";
}

dmoe_status read_info(const GgufFile& f, dmoe_model_info& in) {
  const std::string mt = model_type(f);
  if (mt != "llada2_moe")
    return mfail(DMOE_ERR_UNSUPPORTED, "model type %s has no MoE layers (llada2_moe expected)", mt.c_str());
  uint32_t n_layer, n_embd, n_exp, n_used, n_shared, moe_ff, first_k, norm_topk, cap, block_len, moe_blk;
  float scale;
  dmoe_status s;
  if ((s = get_u32(f, "block_count", true, 0, n_layer)) != DMOE_OK) return s;
  if ((s = get_u32(f, "embedding_length", true, 0, n_embd)) != DMOE_OK) return s;
  if ((s = get_u32(f, "expert_count", false, 0, n_exp)) != DMOE_OK) return s;
  if ((s = get_u32(f, "expert_used_count", false, 0, n_used)) != DMOE_OK) return s;
  if ((s = get_u32(f, "expert_shared_count", false, 0, n_shared)) != DMOE_OK) return s;
  if ((s = get_u32(f, "expert_feed_forward_length", false, 0, moe_ff)) != DMOE_OK) return s;
  if ((s = get_u32(f, "first_k_dense_replace", false, 0, first_k)) != DMOE_OK) return s;
  if ((s = get_u32(f, "norm_topk_prob", false, 1, norm_topk)) != DMOE_OK) return s;
  if ((s = get_u32(f, "expert_capacity", false, 48, cap)) != DMOE_OK) return s;
  if ((s = get_u32(f, "block_length", false, 0, block_len)) != DMOE_OK) return s;
  if ((s = get_u32(f, "moe_block_size", false, block_len ? block_len : 32, moe_blk)) != DMOE_OK) return s;
  if ((s = get_f32(f, "routed_scaling_factor", 1.0f, scale)) != DMOE_OK) return s;
  if (n_exp == 0 || n_used == 0) return mfail(DMOE_ERR_INVALID_ARG, "expert_count / expert_used_count missing or 0");
  if (first_k > n_layer) return mfail(DMOE_ERR_INVALID_ARG, "first_k_dense_replace %u > block_count %u", first_k, n_layer);
  // every MoE block needs at least four tensors of its own: a block count beyond the file's
  // tensor count is corrupt (and would size the layer table from garbage)
  if ((uint64_t)(n_layer - first_k) * 4 > f.n_tensors())
    return mfail(DMOE_ERR_INVALID_ARG, "block_count %u with %zu tensors in the file", n_layer, f.n_tensors());
  in = dmoe_model_info{};
  in.n_layer = (int32_t)n_layer;
  in.first_k_dense = (int32_t)first_k;
  in.n_moe_layers = (int32_t)(n_layer - first_k);
  in.n_embd = n_embd;
  in.n_ff_exp = moe_ff;
  in.n_expert = n_exp;
  in.n_expert_used = n_used;
  in.expert_capacity = cap;
  in.moe_block_size = moe_blk;
  in.routed_scaling = scale;
  in.norm_topk_prob = (int32_t)norm_topk;
  in.n_ff_shexp = n_shared ? -1 : 0;  // from the first layer's shared tensors
  return DMOE_OK;
}

bool expert_type_ok(int32_t t) { return t == DMOE_TYPE_F16 || t == DMOE_TYPE_Q8_0 || t == DMOE_TYPE_Q4_K; }

dmoe_status need(const GgufFile& f, const std::string& name, const GgufTensor*& t) {
  t = f.tensor(name);
  if (!t) return mfail(DMOE_ERR_INVALID_ARG, "tensor not found: %s", name.c_str());
  if (!t->nbytes) return mfail(DMOE_ERR_UNSUPPORTED, "tensor %s: ggml type %d not handled", name.c_str(), t->type);
  return DMOE_OK;
}

dmoe_status check_shape(const GgufTensor* t, std::initializer_list<int64_t> ne) {
  int d = 0;
  bool ok = t->n_dims == (int)ne.size();
  for (int64_t v : ne) ok = ok && t->ne[d++] == v;
  if (ok) return DMOE_OK;
  std::string want, got;
  for (int64_t v : ne) want += (want.empty() ? "" : ", ") + std::to_string(v);
  for (int i = 0; i < t->n_dims; ++i) got += (got.empty() ? "" : ", ") + std::to_string(t->ne[i]);
  return mfail(DMOE_ERR_INVALID_ARG, "tensor %s: ne [%s], expected [%s]", t->name.c_str(), got.c_str(), want.c_str());
}

// block il's layer descriptor (host pointers into the mapping), with the bytes it references
dmoe_status layer_desc(const GgufFile& f, dmoe_model_info& in, int il, dmoe_layer_desc& d, int64_t& bytes) {
  const std::string b = "blk." + std::to_string(il) + ".";
  const int64_t H = in.n_embd, E = in.n_expert, I = in.n_ff_exp;
  const GgufTensor *router, *gate, *up, *down;
  dmoe_status s;
  if ((s = need(f, b + "moe_gate.weight", router)) != DMOE_OK) return s;
  if (router->type != DMOE_TYPE_F32) return mfail(DMOE_ERR_UNSUPPORTED, "%s must be F32", router->name.c_str());
  if ((s = check_shape(router, {H, E})) != DMOE_OK) return s;
  const GgufTensor* bias = f.tensor(b + "moe_gate_bias.weight");
  if (bias) {
    if (bias->type != DMOE_TYPE_F32) return mfail(DMOE_ERR_UNSUPPORTED, "%s must be F32", bias->name.c_str());
    if ((s = check_shape(bias, {E})) != DMOE_OK) return s;
  }
  if ((s = need(f, b + "moe_experts_gate.weight", gate)) != DMOE_OK) return s;
  if ((s = need(f, b + "moe_experts_up.weight", up)) != DMOE_OK) return s;
  if ((s = need(f, b + "moe_experts_down.weight", down)) != DMOE_OK) return s;
  if ((s = check_shape(gate, {H, I, E})) != DMOE_OK || (s = check_shape(up, {H, I, E})) != DMOE_OK ||
      (s = check_shape(down, {I, H, E})) != DMOE_OK)
    return s;
  if (gate->type != up->type || gate->type != down->type || !expert_type_ok(gate->type))
    return mfail(DMOE_ERR_UNSUPPORTED, "block %d: expert stacks of ggml types %d / %d / %d (one of F16, Q8_0, Q4_K)",
                 il, gate->type, up->type, down->type);
  const GgufTensor *sgate = f.tensor(b + "moe_shared_gate.weight"), *sup = nullptr, *sdown = nullptr;
  int64_t Is = 0;
  if (in.n_ff_shexp != 0) {
    if ((s = need(f, b + "moe_shared_gate.weight", sgate)) != DMOE_OK) return s;
    if ((s = need(f, b + "moe_shared_up.weight", sup)) != DMOE_OK) return s;
    if ((s = need(f, b + "moe_shared_down.weight", sdown)) != DMOE_OK) return s;
    Is = sgate->n_dims == 2 ? sgate->ne[1] : 0;
    if ((s = check_shape(sgate, {H, Is})) != DMOE_OK || (s = check_shape(sup, {H, Is})) != DMOE_OK ||
        (s = check_shape(sdown, {Is, H})) != DMOE_OK)
      return s;
    if (sgate->type != sup->type || sgate->type != sdown->type || !expert_type_ok(sgate->type))
      return mfail(DMOE_ERR_UNSUPPORTED, "block %d: shared expert of ggml types %d / %d / %d", il, sgate->type,
                   sup->type, sdown->type);
    if (in.n_ff_shexp < 0) in.n_ff_shexp = Is;
    if (Is != in.n_ff_shexp)
      return mfail(DMOE_ERR_UNSUPPORTED, "block %d: shared expert width %lld, block %d has %lld", il, (long long)Is,
                   in.first_k_dense, (long long)in.n_ff_shexp);
  } else {
    sgate = nullptr;
  }
  if (il == in.first_k_dense) {
    in.expert_type = gate->type;
    in.shared_type = sgate ? sgate->type : gate->type;
  }
  d = dmoe_layer_desc{};
  d.n_embd = H;
  d.n_ff_exp = I;
  d.n_ff_shexp = Is;
  d.n_expert = E;
  d.n_expert_used = in.n_expert_used;
  d.expert_capacity = in.expert_capacity;
  d.moe_block_size = in.moe_block_size;
  d.routed_scaling = in.routed_scaling;
  d.norm_topk_prob = in.norm_topk_prob;
  d.expert_type = gate->type;
  d.shared_type = sgate ? sgate->type : gate->type;
  d.w_gate = gate->data;
  d.w_up = up->data;
  d.w_down = down->data;
  d.sw_gate = sgate ? sgate->data : nullptr;
  d.sw_up = sup ? sup->data : nullptr;
  d.sw_down = sdown ? sdown->data : nullptr;
  d.w_router = reinterpret_cast<const float*>(router->data);
  d.b_router = bias ? reinterpret_cast<const float*>(bias->data) : nullptr;
  bytes = (int64_t)(router->nbytes + (bias ? bias->nbytes : 0) + gate->nbytes + up->nbytes + down->nbytes +
                    (sgate ? sgate->nbytes + sup->nbytes + sdown->nbytes : 0));
  return DMOE_OK;
}

dmoe_status open_and_scan(const char* path, GgufFile& f, dmoe_model_info& in, std::vector<dmoe_layer_desc>& descs) {
  if (!path) return mfail(DMOE_ERR_INVALID_ARG, "null path");
  std::string err;
  if (!f.open(path, err)) return mfail(DMOE_ERR_INVALID_ARG, "%s", err.c_str());
  dmoe_status s = read_info(f, in);
  if (s != DMOE_OK) return s;
  descs.assign((size_t)in.n_layer, dmoe_layer_desc{});
  for (int il = in.first_k_dense; il < in.n_layer; ++il) {
    int64_t bytes = 0;
    if ((s = layer_desc(f, in, il, descs[(size_t)il], bytes)) != DMOE_OK) return s;
    in.moe_bytes += bytes;
  }
  if (in.n_ff_shexp < 0) in.n_ff_shexp = 0;
  return DMOE_OK;
}

}  // namespace

extern "C" {

dmoe_status dmoe_model_inspect(const char* path, dmoe_model_info* info) {
  if (!info) return mfail(DMOE_ERR_INVALID_ARG, "null info");
  try {
    GgufFile f;
    dmoe_model_info in{};
    std::vector<dmoe_layer_desc> descs;
    const dmoe_status s = open_and_scan(path, f, in, descs);
    if (s == DMOE_OK) *info = in;
    return s;
  } catch (const std::exception& e) {  // host allocation failure while reading the file
    return mfail(DMOE_ERR_OOM, "reading %s: %s", path, e.what());
  }
}

dmoe_status dmoe_model_load(const char* path, const dmoe_dist_cfg* dist, dmoe_model** out) {
  if (!out) return mfail(DMOE_ERR_INVALID_ARG, "null output handle");
  *out = nullptr;
  GgufFile f;
  dmoe_model_info in{};
  std::vector<dmoe_layer_desc> descs;
  dmoe_status s;
  try {
    s = open_and_scan(path, f, in, descs);
  } catch (const std::exception& e) {  // host allocation failure while reading the file
    return mfail(DMOE_ERR_OOM, "reading %s: %s", path, e.what());
  }
  if (s != DMOE_OK) return s;
  dmoe_model* m = new dmoe_model();
  m->info = in;
  m->layers.assign((size_t)in.n_layer, nullptr);
  const bool ep = dist && dist->world_size > 1;
  dmoe_layer* first = nullptr;
  for (int il = in.first_k_dense; il < in.n_layer; ++il) {
    dmoe_layer* L = nullptr;
    s = (ep && first) ? dmoe_create_split(&descs[(size_t)il], dist, first, &L)
                      : dmoe_create(&descs[(size_t)il], dist, &L);
    if (s != DMOE_OK) {
      char msg[1200];
      dmoe_last_error(msg, sizeof(msg) - 64);
      const std::string m2 = "block " + std::to_string(il) + ": " + msg;
      dmoe_model_free(m);
      return mfail(s, "%s", m2.c_str());
    }
    m->layers[(size_t)il] = L;
    if (!first) first = L;
  }
  *out = m;
  return DMOE_OK;
}

dmoe_status dmoe_model_get_info(const dmoe_model* m, dmoe_model_info* info) {
  if (!m || !info) return mfail(DMOE_ERR_INVALID_ARG, "null model or info");
  *info = m->info;
  return DMOE_OK;
}

dmoe_layer* dmoe_model_layer(dmoe_model* m, int32_t il) {
  if (!m || il < 0 || il >= (int32_t)m->layers.size()) return nullptr;
  return m->layers[(size_t)il];
}

void dmoe_model_free(dmoe_model* m) {
  if (!m) return;
  // later layers first: their communicators were split from the first one's
  for (size_t i = m->layers.size(); i-- > 0;) dmoe_destroy(m->layers[i]);
  delete m;
}

}  // extern "C"

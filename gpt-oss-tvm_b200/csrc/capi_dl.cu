// capi_dl.cu -- the DLTensor entry points (include/gptoss_b200_dlpack.h):
// every argument is checked (element type, shape, agreement between tensors,
// CUDA device = the current one, dense row-major layout) before the
// plain-pointer entry point of gptoss_b200.h is called.
#include <cstdarg>
#include <cstdio>

#include "../../include/gptoss_b200_dlpack.h"
#include "launch.h"

namespace {

int dl_fail(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return gptoss::set_last_error(-1, buf);
}

enum Dt { kBf16, kF32, kU8, kI32 };

const char* dt_name(Dt d) { return d == kBf16 ? "bfloat16" : d == kF32 ? "float32" : d == kU8 ? "uint8" : "int32"; }

bool dt_is(const DLDataType& t, Dt d) {
  if (t.lanes != 1) return false;
  switch (d) {
    case kBf16: return t.code == kDLBfloat && t.bits == 16;
    case kF32: return t.code == kDLFloat && t.bits == 32;
    case kU8: return t.code == kDLUInt && t.bits == 8;
    case kI32: return t.code == kDLInt && t.bits == 32;
  }
  return false;
}

// The argument checks of one call: the first failure is reported with the
// function and argument names; later checks are skipped.
struct Checker {
  const char* fn;
  int rc = 0;
  int dev = -1;

  explicit Checker(const char* f) : fn(f) {
    if (cudaGetDevice(&dev) != cudaSuccess) {
      (void)cudaGetLastError();
      dev = -1;
    }
  }

  // tensor t: element type d, ndim dims with the given sizes (-1: any)
  bool tensor(const char* name, const DLTensor* t, Dt d, int ndim, const int64_t* shape) {
    if (rc) return false;
    if (!t) { rc = dl_fail("%s: %s is NULL", fn, name); return false; }
    if (t->device.device_type != kDLCUDA || t->device.device_id != dev) {
      rc = dl_fail("%s: %s must be on the current CUDA device (cuda:%d), got device type %d id %d", fn, name, dev,
                   (int)t->device.device_type, (int)t->device.device_id);
      return false;
    }
    if (!dt_is(t->dtype, d)) {
      rc = dl_fail("%s: %s must be %s (got type code %d, %d bits, %d lanes)", fn, name, dt_name(d),
                   (int)t->dtype.code, (int)t->dtype.bits, (int)t->dtype.lanes);
      return false;
    }
    if (t->ndim != ndim) { rc = dl_fail("%s: %s must have %d dimensions (got %d)", fn, name, ndim, t->ndim); return false; }
    for (int i = 0; i < ndim; ++i) {
      if (shape[i] >= 0 && t->shape[i] != shape[i]) {
        rc = dl_fail("%s: %s dimension %d must be %lld (got %lld)", fn, name, i, (long long)shape[i],
                     (long long)t->shape[i]);
        return false;
      }
    }
    if (t->strides) {
      int64_t expect = 1;
      for (int i = ndim - 1; i >= 0; --i) {
        if (t->shape[i] != 1 && t->strides[i] != expect) {
          rc = dl_fail("%s: %s must be dense row-major (dimension %d has stride %lld, expected %lld)", fn, name, i,
                       (long long)t->strides[i], (long long)expect);
          return false;
        }
        expect *= t->shape[i];
      }
    }
    return true;
  }
};

template <class T>
T* ptr(const DLTensor* t) {
  return t ? (T*)((char*)t->data + t->byte_offset) : nullptr;
}

int64_t dim(const DLTensor* t, int i) { return t->shape[i]; }

}  // namespace

extern "C" int gptoss_moe_weights_init_dl(gptoss_moe_weights* w, const DLTensor* norm_weight,
                                          const DLTensor* gate_weight, const DLTensor* gate_bias,
                                          const DLTensor* mlp1_blocks, const DLTensor* mlp1_scales,
                                          const DLTensor* mlp1_bias, const DLTensor* mlp2_blocks,
                                          const DLTensor* mlp2_scales, const DLTensor* mlp2_bias, int32_t top_k,
                                          float swiglu_limit, float rms_eps, int32_t expert_offset, void* stream) {
  const char* fn = "gptoss_moe_weights_init_dl";
  if (!w) return dl_fail("%s: w is NULL", fn);
  if (!gate_weight || gate_weight->ndim != 2 || !mlp1_blocks || mlp1_blocks->ndim != 4 || !mlp2_blocks ||
      mlp2_blocks->ndim != 4)
    return dl_fail("%s: gate_weight must be [E, H], mlp1_blocks and mlp2_blocks [El, rows, groups, 16]", fn);
  const int64_t E = dim(gate_weight, 0), H = dim(gate_weight, 1), El = dim(mlp1_blocks, 0);
  const int64_t I = dim(mlp1_blocks, 1) / 2;
  if (H % 32 || I % 32 || dim(mlp1_blocks, 1) % 2 || E <= 0 || El <= 0)
    return dl_fail("%s: hidden and intermediate sizes must be multiples of 32", fn);
  if (expert_offset < 0 || expert_offset + El > E || top_k < 1 || top_k > 8 || top_k > E)
    return dl_fail("%s: experts [%d, %lld) outside the router's %lld, or top_k %d out of range", fn, expert_offset,
                   (long long)(expert_offset + El), (long long)E, top_k);
  Checker c(fn);
  const int64_t s_norm[1] = {H}, s_gw[2] = {E, H}, s_gb[1] = {E};
  const int64_t s_b1[4] = {El, 2 * I, H / 32, 16}, s_s1[3] = {El, 2 * I, H / 32}, s_bias1[2] = {El, 2 * I};
  const int64_t s_b2[4] = {El, H, I / 32, 16}, s_s2[3] = {El, H, I / 32}, s_bias2[2] = {El, H};
  c.tensor("norm_weight", norm_weight, kBf16, 1, s_norm);
  c.tensor("gate_weight", gate_weight, kBf16, 2, s_gw);
  c.tensor("gate_bias", gate_bias, kBf16, 1, s_gb);
  c.tensor("mlp1_weight_blocks", mlp1_blocks, kU8, 4, s_b1);
  c.tensor("mlp1_weight_scales", mlp1_scales, kU8, 3, s_s1);
  c.tensor("mlp1_bias", mlp1_bias, kBf16, 2, s_bias1);
  c.tensor("mlp2_weight_blocks", mlp2_blocks, kU8, 4, s_b2);
  c.tensor("mlp2_weight_scales", mlp2_scales, kU8, 3, s_s2);
  c.tensor("mlp2_bias", mlp2_bias, kBf16, 2, s_bias2);
  if (c.rc) return c.rc;
  gptoss_moe_weights v = {};
  v.num_experts = (int32_t)E;
  v.num_local_experts = (int32_t)El;
  v.expert_offset = expert_offset;
  v.hidden = (int32_t)H;
  v.intermediate = (int32_t)I;
  v.top_k = top_k;
  v.swiglu_alpha = 1.702f;
  v.swiglu_limit = swiglu_limit;
  v.rms_eps = rms_eps;
  v.norm_weight = ptr<const uint16_t>(norm_weight);
  v.gate_weight = ptr<const uint16_t>(gate_weight);
  v.gate_bias = ptr<const uint16_t>(gate_bias);
  v.mlp1_blocks = ptr<const uint8_t>(mlp1_blocks);
  v.mlp1_scales = ptr<const uint8_t>(mlp1_scales);
  v.mlp1_bias = ptr<const uint16_t>(mlp1_bias);
  v.mlp2_blocks = ptr<const uint8_t>(mlp2_blocks);
  v.mlp2_scales = ptr<const uint8_t>(mlp2_scales);
  v.mlp2_bias = ptr<const uint16_t>(mlp2_bias);
  v.flags = 0;
  const int rc = gptoss_moe_weights_prepare(&v, stream);
  if (rc) return rc;
  *w = v;
  return 0;
}

extern "C" int gptoss_moe_forward_dl(const DLTensor* x, const gptoss_moe_weights* w, gptoss_moe_workspace* ws,
                                     DLTensor* out, void* stream) {
  const char* fn = "gptoss_moe_forward_dl";
  if (!w || !ws) return dl_fail("%s: w and ws are required", fn);
  if (!x || x->ndim < 1 || x->ndim > 4) return dl_fail("%s: x must have 1 to 4 dimensions", fn);
  Checker c(fn);
  int64_t shape[4];
  int64_t M = 1;
  for (int i = 0; i < x->ndim; ++i) shape[i] = x->shape[i];
  shape[x->ndim - 1] = w->hidden;
  for (int i = 0; i + 1 < x->ndim; ++i) M *= x->shape[i];
  c.tensor("x", x, kBf16, x->ndim, shape);
  for (int i = 0; i < x->ndim; ++i) shape[i] = x->shape[i];
  c.tensor("out", out, kBf16, x->ndim, shape);
  if (c.rc) return c.rc;
  return gptoss_moe_forward(ptr<const uint16_t>(x), M, w, ws, ptr<uint16_t>(out), stream);
}

extern "C" int gptoss_attn_prefill_dl(const DLTensor* q, const DLTensor* k, const DLTensor* v, const DLTensor* sinks,
                                      int32_t window, float sm_scale, DLTensor* o, DLTensor* lse, void* stream) {
  const char* fn = "gptoss_attn_prefill_dl";
  if (!q || !k || (q->ndim != 3 && q->ndim != 4) || k->ndim != q->ndim)
    return dl_fail("%s: q and k must be [S, heads, 64] (or [1, S, heads, 64])", fn);
  const int b = q->ndim - 3;  // a leading batch dimension of 1
  if (b && (q->shape[0] != 1 || k->shape[0] != 1)) return dl_fail("%s: the batch dimension must be 1", fn);
  const int64_t Sq = q->shape[b], Hq = q->shape[b + 1], Skv = k->shape[b], Hkv = k->shape[b + 1];
  Checker c(fn);
  int64_t sq[4] = {1, Sq, Hq, 64}, sk[4] = {1, Skv, Hkv, 64};
  c.tensor("q", q, kBf16, q->ndim, sq + (1 - b));
  c.tensor("k", k, kBf16, q->ndim, sk + (1 - b));
  c.tensor("v", v, kBf16, q->ndim, sk + (1 - b));
  c.tensor("o", o, kBf16, q->ndim, sq + (1 - b));
  const int64_t sh[1] = {Hq};
  if (sinks) c.tensor("sinks", sinks, kBf16, 1, sh);
  const int64_t sl[3] = {1, Sq, Hq};
  if (lse) c.tensor("lse", lse, kF32, 2 + b, sl + (1 - b));
  if (c.rc) return c.rc;
  return gptoss_attn_prefill(ptr<const uint16_t>(q), ptr<const uint16_t>(k), ptr<const uint16_t>(v),
                             ptr<const uint16_t>(sinks), Sq, Skv, (int32_t)Hq, (int32_t)Hkv, 64, window, sm_scale,
                             ptr<uint16_t>(o), ptr<float>(lse), stream);
}

extern "C" int gptoss_attn_decode_dl(const DLTensor* q, const DLTensor* k_cache, const DLTensor* v_cache,
                                     const DLTensor* kv_len, int32_t window, float sm_scale, const DLTensor* sinks,
                                     DLTensor* scratch, DLTensor* o, DLTensor* lse, void* stream) {
  const char* fn = "gptoss_attn_decode_dl";
  if (!q || q->ndim != 3 || !k_cache || k_cache->ndim != 4)
    return dl_fail("%s: q must be [B, Hq, 64] and the caches [B, max_len, Hkv, 64]", fn);
  const int64_t B = q->shape[0], Hq = q->shape[1], L = k_cache->shape[1], Hkv = k_cache->shape[2];
  Checker c(fn);
  const int64_t sq[3] = {B, Hq, 64}, sc[4] = {B, L, Hkv, 64}, sb[1] = {B}, sh[1] = {Hq}, sl[2] = {B, Hq};
  c.tensor("q", q, kBf16, 3, sq);
  c.tensor("k_cache", k_cache, kBf16, 4, sc);
  c.tensor("v_cache", v_cache, kBf16, 4, sc);
  c.tensor("kv_len", kv_len, kI32, 1, sb);
  c.tensor("o", o, kBf16, 3, sq);
  if (sinks) c.tensor("sinks", sinks, kBf16, 1, sh);
  if (lse) c.tensor("lse", lse, kF32, 2, sl);
  const int64_t any1[1] = {-1};
  if (scratch) c.tensor("scratch", scratch, kF32, 1, any1);
  if (c.rc) return c.rc;
  const int64_t scratch_bytes = scratch ? scratch->shape[0] * 4 : 0;
  return gptoss_attn_decode(ptr<const uint16_t>(q), ptr<const uint16_t>(k_cache), ptr<const uint16_t>(v_cache),
                            ptr<const int32_t>(kv_len), B, L, (int32_t)Hq, (int32_t)Hkv, 64, window, sm_scale,
                            ptr<const uint16_t>(sinks), ptr<float>(scratch), scratch_bytes, ptr<uint16_t>(o),
                            ptr<float>(lse), stream);
}

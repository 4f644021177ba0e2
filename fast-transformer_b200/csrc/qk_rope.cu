// Fused per-head Q/K RMSNorm + rotate-half RoPE + KV-cache append (sm_100a).
//
// Arithmetic and cast points follow the reference kernel `_qk_rope_cache`
// (engine/kernels/qk_rope.py:13-84):
//   inv  = 1 / sqrt(mean(x^2) + eps)            fp32 (:34-36)
//   n    = bf16(x * inv); w = bf16(n * gain)    (:45-48)
//   rot  = [-w[D/2:], w[:D/2]]                  (:49)
//   out  = bf16(bf16(w * cos) + bf16(rot * sin)) both products rounded (:62-66)
// Q heads go to a token-major [B, T, Hq, D] buffer (:67-68); K heads and the matching V
// heads (copied unchanged, :82-84) go to the cache slot of each token (:70-81).
// Split-K fp32 inputs are summed in split order, then rounded (merged.py:37-45).
//
// One warp per (token row, head); each lane owns D/32 consecutive dims, so the
// rotate-half partner of a lane's dims sits in lane ^ 16 and one shuffle pairs them.
#include "common.cuh"
#include "rope_math.cuh"

namespace fb {
namespace rope {

struct Params {
  const void* packed;
  int splits;
  const __nv_bfloat16* q_weight;
  const __nv_bfloat16* k_weight;
  float q_eps, k_eps;
  const __nv_bfloat16* cos;
  const __nv_bfloat16* sin;
  const int64_t* position;
  const int64_t* phases;
  __nv_bfloat16* query;
  __nv_bfloat16* keys;
  __nv_bfloat16* values;
  int batch, tokens, q_heads, kv_heads, capacity, mode, table;
  unsigned* err;
};

// Loads E consecutive packed values at element offset `off` as fp32 holding bf16 values.
template <int E>
__device__ __forceinline__ void load_packed(const Params& p, size_t off, size_t split_stride,
                                            float (&x)[E]) {
  load_packed_values<E>(p.packed, p.splits, off, split_stride, x);
}

template <int D>
__global__ void __launch_bounds__(128) qk_rope_kernel(const Params p) {
  constexpr int E = D / 32;
  const int warp_global = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int heads = p.q_heads + p.kv_heads;
  const int rows = p.batch * p.tokens;
  if (warp_global >= rows * heads) return;  // a CTA's spare warps touch nothing
  const int row = warp_global / heads;
  const int head = warp_global % heads;
  const int b = row / p.tokens;
  const int t = row % p.tokens;
  const int width = (p.q_heads + 2 * p.kv_heads) * D;
  const size_t split_stride = static_cast<size_t>(rows) * width;
  const int d0 = lane * E;

  const bool is_q = head < p.q_heads;
  const int kvh = head - p.q_heads;
  // the norm gains are never written while decoding: load them before the dependency wait
  const __nv_bfloat16* gain = is_q ? p.q_weight : p.k_weight;
  float gw[E];
  load_bf16<E>(gain + d0, gw);
  pdl_wait();
  pdl_trigger();
  // Every other global read is issued up front (the V head before any store that could
  // alias it).
  float x[E], v[E];
  load_packed<E>(p, static_cast<size_t>(row) * width + head * D + d0, split_stride, x);
  if (!is_q)
    load_packed<E>(p, static_cast<size_t>(row) * width + (p.q_heads + p.kv_heads + kvh) * D + d0,
                   split_stride, v);
  long long pos_base = 0;
  if (p.mode == 2)
    pos_base = __ldg(p.position + b);
  else if (p.mode == 0)
    pos_base = __ldg(p.position);
  long long phase;
  if (p.table) {
    // whole tables: the phase row is the token's position (plus its verify-block phase)
    phase = pos_base + (p.phases != nullptr ? p.phases[row] : t);
  } else {
    phase = p.mode == 2 ? row : t;
  }
  __nv_bfloat16 outv[E];
  norm_rope<D>(x, gw, is_q ? p.q_eps : p.k_eps, p.cos + phase * D + d0, p.sin + phase * D + d0, lane, outv);
  if (is_q) {
    __nv_bfloat16* dst = p.query + (static_cast<size_t>(row) * p.q_heads + head) * D + d0;
#pragma unroll
    for (int e = 0; e < E; ++e) dst[e] = outv[e];
    return;
  }
  const long long pos = p.mode == 1 ? t : pos_base + t;
  if (pos < 0 || pos >= p.capacity) {
    if (lane == 0) raise_error(p.err, kErrBadShape);
    return;
  }
  const size_t slot = ((static_cast<size_t>(b) * p.kv_heads + kvh) * p.capacity + pos) * D + d0;
#pragma unroll
  for (int e = 0; e < E; ++e) p.keys[slot + e] = outv[e];
#pragma unroll
  for (int e = 0; e < E; ++e) p.values[slot + e] = __float2bfloat16_rn(v[e]);
}

}  // namespace rope
}  // namespace fb

using namespace fb;

extern "C" int fb_qk_norm_rope_append(const void* packed, int packed_splits, const void* q_weight,
                                      const void* k_weight, float q_eps, float k_eps,
                                      const void* cos, const void* sin, const int64_t* position,
                                      const int64_t* phases, void* query, void* keys, void* values,
                                      int batch, int tokens, int q_heads, int kv_heads,
                                      int head_dim, int capacity, int mode, int table,
                                      void* stream) {
  if (!packed || !q_weight || !k_weight || !cos || !sin || !position || !query || !keys ||
      !values)
    return FB_ERR_ARG;
  if (batch <= 0 || tokens <= 0 || q_heads <= 0 || kv_heads <= 0 || capacity <= 0 ||
      packed_splits < 0)
    return FB_ERR_ARG;
  if (mode < 0 || mode > 2 || (table && mode == 1)) return FB_ERR_ARG;
  if (head_dim != 64 && head_dim != 128) return FB_ERR_SHAPE;
  if (tokens > capacity) return FB_ERR_SHAPE;
  rope::Params p;
  p.packed = packed;
  p.splits = packed_splits;
  p.q_weight = static_cast<const __nv_bfloat16*>(q_weight);
  p.k_weight = static_cast<const __nv_bfloat16*>(k_weight);
  p.q_eps = q_eps;
  p.k_eps = k_eps;
  p.cos = static_cast<const __nv_bfloat16*>(cos);
  p.sin = static_cast<const __nv_bfloat16*>(sin);
  p.position = position;
  p.phases = phases;
  p.query = static_cast<__nv_bfloat16*>(query);
  p.keys = static_cast<__nv_bfloat16*>(keys);
  p.values = static_cast<__nv_bfloat16*>(values);
  p.batch = batch;
  p.tokens = tokens;
  p.q_heads = q_heads;
  p.kv_heads = kv_heads;
  p.capacity = capacity;
  p.mode = mode;
  p.table = table ? 1 : 0;
  p.err = error_word();
  const long long warps = static_cast<long long>(batch) * tokens * (q_heads + kv_heads);
  const int blocks = static_cast<int>((warps + 3) / 4);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (head_dim == 128) return launch_ex(rope::qk_rope_kernel<128>, dim3(blocks), dim3(128), 0, s, 1, p);
  return launch_ex(rope::qk_rope_kernel<64>, dim3(blocks), dim3(128), 0, s, 1, p);
}

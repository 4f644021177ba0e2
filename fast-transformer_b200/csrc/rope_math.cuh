// Per-head QK-RMSNorm + rotate-half RoPE on one warp, shared by the stand-alone kernel
// (qk_rope.cu) and the qkv projection's fused epilogue (linear.cu).
//
// Arithmetic and cast points of the reference kernel `_qk_rope_cache`
// (engine/kernels/qk_rope.py:34-66):
//   inv  = 1 / sqrt(mean(x^2) + eps)            fp32, the sum of squares in the reference's
//                                               eager (torch CPU) order: bit-exact K and Q
//   n    = bf16(x * inv); w = bf16(n * gain)
//   rot  = [-w[D/2:], w[:D/2]]
//   out  = bf16(bf16(w * cos) + bf16(rot * sin)) both products rounded
// Lane l holds dims [l*E, l*E + E), E = D/32, so the rotate-half partner of a lane's dims
// sits in lane ^ 16.
#pragma once

#include "common.cuh"

namespace fb {
namespace rope {

// Loads E consecutive bf16 values at `src` (8- or 4-byte aligned) as fp32.
template <int E>
__device__ __forceinline__ void load_bf16(const __nv_bfloat16* src, float (&x)[E]) {
  if constexpr (E == 4) {
    const uint2 w = __ldg(reinterpret_cast<const uint2*>(src));
    x[0] = bf16_lo(w.x);
    x[1] = bf16_hi(w.x);
    x[2] = bf16_lo(w.y);
    x[3] = bf16_hi(w.y);
  } else {
    const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(src));
    x[0] = bf16_lo(w);
    x[1] = bf16_hi(w);
  }
}

// E consecutive values at element `off` of the packed qkv projection output, as fp32 holding
// bf16 values: bf16 [rows, width] when splits == 0, else fp32 split-K partials [splits, rows,
// width] (slab stride `split_stride`) summed in split order and rounded to bf16
// (engine/kernels/merged.py:37-45). Up to kBatch slabs' loads are in flight before their
// in-order adds (the batch changes only the load schedule, not the sum). The input was
// written by an earlier kernel: plain / L2 loads, not __ldg.
template <int E, int kBatch = 16>
__device__ __forceinline__ void load_packed_values(const void* packed, int splits, size_t off, size_t split_stride,
                                                   float (&x)[E]) {
  if (splits == 0) {
    const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(packed) + off;
    if constexpr (E == 4) {
      const uint2 w = *reinterpret_cast<const uint2*>(src);
      x[0] = bf16_lo(w.x);
      x[1] = bf16_hi(w.x);
      x[2] = bf16_lo(w.y);
      x[3] = bf16_hi(w.y);
    } else {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(src);
      x[0] = bf16_lo(w);
      x[1] = bf16_hi(w);
    }
    return;
  }
  const float* src = static_cast<const float*>(packed) + off;
  for (int s0 = 0; s0 < splits; s0 += kBatch) {
    float y[kBatch][E];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      if (s0 + j < splits) {
        const float* q = src + (s0 + j) * split_stride;
        if constexpr (E == 4) {
          const float4 a = __ldcg(reinterpret_cast<const float4*>(q));
          y[j][0] = a.x;
          y[j][1] = a.y;
          y[j][2] = a.z;
          y[j][3] = a.w;
        } else {
          const float2 a = __ldcg(reinterpret_cast<const float2*>(q));
          y[j][0] = a.x;
          y[j][1] = a.y;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      if (s0 + j == 0) {
#pragma unroll
        for (int e = 0; e < E; ++e) x[e] = y[0][e];
      } else if (s0 + j < splits) {
#pragma unroll
        for (int e = 0; e < E; ++e) x[e] += y[j][e];
      }
    }
  }
#pragma unroll
  for (int e = 0; e < E; ++e) x[e] = bf16_round(x[e]);
}

// Sum of the squares of one head's D values (lane l holds dims [l*E, l*E + E)), added in the
// order of torch's CPU sum kernel for a contiguous fp32 row, which is the order the
// reference's eager `x.pow(2).mean(-1)` uses (agent/local_cpu/shim/references.py:155):
//   - the row is read as 8-wide vectors v_0 .. v_{D/8-1};
//   - four interleaved vector accumulators, a_k = ((v_k + v_{k+4}) + v_{k+8}) + ...;
//   - then ((a_0 + a_1) + a_2) + a_3, lane-wise;
//   - then its 8 lanes in index order.
// Every product and sum is rounded on its own (no fused multiply-add), so the result has the
// bits torch computes on the host. Every lane of the warp must call it; all lanes return the
// total.
template <int D>
__device__ __forceinline__ float sum_squares_host_order(const float (&x)[D / 32]) {
  constexpr int E = D / 32;      // values per lane
  constexpr int V = 8 / E;       // lanes per 8-wide vector
  constexpr int R = D / 32;      // vectors per accumulator: (D / 8) / 4
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  float sq[E], acc[E], vec[E];
#pragma unroll
  for (int e = 0; e < E; ++e) sq[e] = __fmul_rn(x[e], x[e]);
  // lanes [0, 4V) hold vector k = lane / V; accumulator k adds vectors k, k+4, ... in order
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = sq[e];
#pragma unroll
  for (int r = 1; r < R; ++r) {
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] = __fadd_rn(acc[e], __shfl_down_sync(0xffffffffu, sq[e], 4 * V * r));
  }
  // lanes [0, V) combine the four accumulators in order
#pragma unroll
  for (int e = 0; e < E; ++e) vec[e] = acc[e];
#pragma unroll
  for (int k = 1; k < 4; ++k) {
#pragma unroll
    for (int e = 0; e < E; ++e) vec[e] = __fadd_rn(vec[e], __shfl_down_sync(0xffffffffu, acc[e], V * k));
  }
  // the 8 vector lanes, held E at a time by lanes 0 .. V-1, in index order
  float total = 0.f;
#pragma unroll
  for (int h = 0; h < V; ++h) {
#pragma unroll
    for (int e = 0; e < E; ++e) total = __fadd_rn(total, __shfl_sync(0xffffffffu, vec[e], h));
  }
  return total;
}

// x: this lane's E values of one head (fp32 holding bf16 values); gw: the matching norm gains;
// cs/sn: the cos/sin table row of the token's phase, offset to this lane's first dim.
// Every lane of the warp must call it (shuffle reduction, one partner exchange).
template <int D>
__device__ __forceinline__ void norm_rope(const float (&x)[D / 32], const float (&gw)[D / 32], float eps,
                                          const __nv_bfloat16* cs, const __nv_bfloat16* sn, int lane,
                                          __nv_bfloat16 (&out)[D / 32]) {
  constexpr int E = D / 32;
  const float ss = sum_squares_host_order<D>(x);
  // mean = sum / D, then 1 / sqrt(mean + eps), each correctly rounded (torch.rsqrt on the
  // host divides 1 by a correctly rounded square root)
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(D)), eps)));
  float w[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float n = bf16_round(x[e] * inv);
    w[e] = bf16_round(n * gw[e]);
  }
  float partner[E];
#pragma unroll
  for (int e = 0; e < E; ++e) partner[e] = __shfl_xor_sync(0xffffffffu, w[e], 16);
  const bool low_half = lane < 16;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float rot = low_half ? -partner[e] : partner[e];
    const float direct = bf16_round(w[e] * __bfloat162float(cs[e]));
    const float turn = bf16_round(rot * __bfloat162float(sn[e]));
    out[e] = __float2bfloat16_rn(direct + turn);
  }
}

}  // namespace rope
}  // namespace fb

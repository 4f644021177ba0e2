// Split-KV GQA decode attention for sm_100a.
//
// Semantics follow the reference's `_decode_partials` + `_decode_merge`
// (engine/kernels/decode_attention.py:31-127): for each (row b, KV head h) the G query
// heads of that group attend to cache slots [0, len_b), len_b = position + 1; scores are
// fp32 dot products scaled by scale*log2(e), softmax uses exp2 with a running maximum,
// probabilities are rounded to bf16 before the P*V product (:90) while the denominator
// sums the unrounded fp32 probabilities (:83), and splits are merged with a
// log-sum-exp combine (:119-127).
//
// B200 design (not a translation of the Triton kernel):
//  * Work unit = one 64-token tile of one (row, KV head). All valid tiles of all pairs
//    form one sequence (row-major, then head, then tile); a persistent grid of `ctas`
//    CTAs takes equal contiguous slices of it, so ragged lengths balance across SMs.
//    Consecutive tiles of the same pair inside a CTA are one "run" with one online
//    softmax state; a run that covers a whole pair writes the final output directly.
//  * Warp 4 (one elected lane) streams K and V tiles with 2-D TMA loads
//    (CU_TENSOR_MAP_SWIZZLE_128B, no multicast) into an NS-stage mbarrier ring.
//  * Warps 0-3 each take 16 tokens of a tile. Scores are computed transposed,
//    S^T[16 tok x 8 heads] = K * Q^T, with mma.sync m16n8k16 (Q^T held in registers for
//    the whole run), the probabilities are transposed in registers (movmatrix) and
//    O^T[D x 8] += V^T * P^T accumulates in registers. The swizzled layout makes every
//    ldmatrix conflict-free.
//  * Partials of runs that do not cover their pair go to slot (cta + pair) of the
//    workspace; the combine kernel re-derives which CTAs touched each pair from the same
//    integer partition, so no counters or atomics are needed and results are
//    deterministic.
#include <mutex>

#include "common.cuh"

namespace fb {
namespace attn {

constexpr int kTile = 64;          // tokens per pipeline stage
constexpr int kConsumerWarps = 4;  // 16 tokens each
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kMaxBatch = 1024;
constexpr int kHeadsPad = 8;  // query heads per KV head, padded to the mma N
constexpr int kMaxCtas = 512;  // persistent CTAs (runs per pair are bounded by this)

struct Params {
  const __nv_bfloat16* q;  // [B, Hq, D]
  const int64_t* position;
  int per_row;
  __nv_bfloat16* out;  // [B, Hq, D]
  float* acc;          // [slots, G, D]
  float2* stats;       // [slots, G] (max, denominator)
  int* counters;       // [B * Hkv] runs finished per pair (fused merge); nullptr: no merge
  int batch, q_heads, kv_heads, groups, capacity, ctas;
  float scale_log2;
  unsigned* err;
};

// Valid length of row b: position + 1 clamped into [0, capacity].
__device__ __forceinline__ int row_length(const int64_t* position, int per_row, int b,
                                          int capacity) {
  long long p = position[per_row ? b : 0];
  long long n = p + 1;
  if (n < 0) n = 0;
  if (n > capacity) n = capacity;
  return static_cast<int>(n);
}

__device__ __forceinline__ int tiles_of(int len) { return (len + kTile - 1) / kTile; }

// First tile of CTA i in a sequence of T tiles split over G CTAs.
__device__ __forceinline__ long long slice_start(long long T, int i, int G) {
  return (T * i) / G;
}
// The CTA whose slice contains tile t (largest i with slice_start(i) <= t).
__device__ __forceinline__ int slice_owner(long long T, long long t, int G) {
  return static_cast<int>(((t + 1) * G - 1) / T);
}

// Merge the runs of CTAs lo..hi on one (row, KV head) pair into its bf16 output:
// out = sum_i acc_i * exp2(m_i - M) / sum_i l_i * exp2(m_i - M) per query head, the runs
// taken in increasing CTA order (deterministic). A CTA in [lo, hi] whose slice is empty
// wrote nothing and gets weight 0. Partials are read through L2 (ld.global.cg): they were
// written by other CTAs of this launch moments ago.
//
// A pair of at most kMergeRuns runs (the common case: a pair shared by neighbouring slices)
// takes one L2 round trip: each thread owns outputs tid, tid + Threads, ... and loads every
// run's accumulator for them together with the (m, l) of each output's head, with no block
// barrier. Longer pairs resolve the runs' weights once into shared memory (warp per head),
// then sweep the accumulators.
constexpr int kMergeRuns = 4;

template <int D, int Threads>
__device__ void merge_short_pair(const Params& p, int pair, int lo, int runs, long long T, int tid) {
  constexpr int kOut = (kHeadsPad * D + Threads - 1) / Threads;  // outputs per thread at most
  const int G = p.groups;
  const int outputs = G * D;
  const bool all_nonempty = T >= p.ctas;
  const int b = pair / p.kv_heads, h = pair % p.kv_heads;
  __nv_bfloat16* out = p.out + (static_cast<size_t>(b) * p.q_heads + h * G) * D;
  const float2* st0 = p.stats + static_cast<size_t>(lo + pair) * G;     // run r, head g: st0[r * G + g]
  const float* acc0 = p.acc + static_cast<size_t>(lo + pair) * outputs;  // run r, output e: acc0[r * G * D + e]
  bool valid[kMergeRuns];
  float2 sv[kMergeRuns][kOut];
  float av[kMergeRuns][kOut];
#pragma unroll
  for (int r = 0; r < kMergeRuns; ++r) {
    valid[r] = r < runs && (all_nonempty || slice_start(T, lo + r, p.ctas) < slice_start(T, lo + r + 1, p.ctas));
#pragma unroll
    for (int k = 0; k < kOut; ++k) {
      const int e = tid + k * Threads;
      const bool on = valid[r] && e < outputs;
      sv[r][k] = on ? __ldcg(st0 + r * G + e / D) : make_float2(-INFINITY, 0.f);
      av[r][k] = on ? __ldcg(acc0 + static_cast<size_t>(r) * outputs + e) : 0.f;
    }
  }
#pragma unroll
  for (int k = 0; k < kOut; ++k) {
    const int e = tid + k * Threads;
    float M = -INFINITY;
#pragma unroll
    for (int r = 0; r < kMergeRuns; ++r) M = fmaxf(M, sv[r][k].x);
    const float piv = M == -INFINITY ? 0.f : M;
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int r = 0; r < kMergeRuns; ++r)
      if (valid[r]) {
        const float w = exp2f(sv[r][k].x - piv);
        L += sv[r][k].y * w;
        if (w != 0.f) O += av[r][k] * w;
      }
    if (e < outputs) out[e] = __float2bfloat16_rn(O / L);
  }
}

template <int D, int Threads, typename Bar>
__device__ void merge_pair(const Params& p, int pair, int lo, int hi, long long T, int tid, float* s_w,
                           float* s_den, Bar bar) {
  const int runs = hi - lo + 1;
  if (runs <= kMergeRuns) {
    merge_short_pair<D, Threads>(p, pair, lo, runs, T, tid);
    return;
  }
  const int threads = Threads;
  const int G = p.groups;
  const int warp = tid >> 5, lane = tid & 31, warps = threads >> 5;
  // With at least one tile per CTA every slice is non-empty: skip the 64-bit tests.
  const bool all_nonempty = T >= p.ctas;
  for (int g = warp; g < G; g += warps) {
    float M = -INFINITY;
    for (int i = lane; i < runs; i += 32)
      if (all_nonempty || slice_start(T, lo + i, p.ctas) < slice_start(T, lo + i + 1, p.ctas))
        M = fmaxf(M, __ldcg(&p.stats[static_cast<size_t>(lo + i + pair) * G + g].x));
    M = warp_max(M);
    const float piv = M == -INFINITY ? 0.f : M;
    float L = 0.f;
    for (int i = lane; i < runs; i += 32) {
      float w = 0.f;
      if (all_nonempty || slice_start(T, lo + i, p.ctas) < slice_start(T, lo + i + 1, p.ctas)) {
        const float2 st = __ldcg(&p.stats[static_cast<size_t>(lo + i + pair) * G + g]);
        w = exp2f(st.x - piv);
        L += st.y * w;
      }
      s_w[i * kHeadsPad + g] = w;
    }
    L = warp_sum(L);
    if (lane == 0) s_den[g] = L;
  }
  bar();
  const int b = pair / p.kv_heads, h = pair % p.kv_heads;
  __nv_bfloat16* out = p.out + (static_cast<size_t>(b) * p.q_heads + h * G) * D;
  constexpr int kBatch = 8;  // run loads in flight before their in-order adds
  for (int e = tid; e < G * D; e += threads) {
    const int g = e / D, d = e % D;
    const float* acc = p.acc + (static_cast<size_t>(lo + pair) * G + g) * D + d;
    const size_t stride = static_cast<size_t>(G) * D;
    float O = 0.f;
    for (int i0 = 0; i0 < runs; i0 += kBatch) {
      float a[kBatch], w[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        w[j] = i0 + j < runs ? s_w[(i0 + j) * kHeadsPad + g] : 0.f;
        a[j] = w[j] != 0.f ? __ldcg(acc + (i0 + j) * stride) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < kBatch; ++j)
        if (w[j] != 0.f) O += a[j] * w[j];
    }
    out[e] = __float2bfloat16_rn(O / s_den[g]);
  }
}

// One consumer warp's running state on one (row, KV head) pair: Q^T fragments, O^T
// accumulators and the online-softmax max/denominator of its two head columns.
template <int D>
struct WarpAcc {
  uint32_t qb[D / 16][2];
  float o[D / 16][4];
  float m0, m1, l0, l1;
};

// Loads query heads h*G..h*G+G-1 of row b as the B operand (heads past G read as zero) and
// clears the running state.
template <int D>
__device__ __forceinline__ void start_pair(WarpAcc<D>& a, const Params& p, int b, int h, int lane) {
  const int g = lane >> 2, c = lane & 3, G = p.groups;
  const bool live = g < G;
  const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
      p.q + (static_cast<size_t>(b) * p.q_heads + h * G + (live ? g : 0)) * D);
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    a.qb[kk][0] = live ? __ldg(qrow + (kk * 16 + 2 * c) / 2) : 0u;
    a.qb[kk][1] = live ? __ldg(qrow + (kk * 16 + 8 + 2 * c) / 2) : 0u;
  }
#pragma unroll
  for (int i = 0; i < D / 16; ++i) a.o[i][0] = a.o[i][1] = a.o[i][2] = a.o[i][3] = 0.f;
  a.m0 = a.m1 = -INFINITY;
  a.l0 = a.l1 = 0.f;
}

// One 64-token K/V tile (128-byte swizzled, D/64 boxes of 64 columns) starting at token
// tile_start of a row with `len` valid tokens: this warp's 16 tokens, S^T = K * Q^T, the
// online softmax over tokens, and O^T += V^T * P^T with P rounded to bf16.
template <int D>
__device__ __forceinline__ void attend_tile(WarpAcc<D>& a, uint8_t* kt, uint8_t* vt, int tile_start, int len,
                                            int warp, int lane, float sl2) {
  constexpr int kBoxes = D / 64;
  constexpr int kKSteps = D / 16;
  const int g = lane >> 2;
  const int slice = tile_start + warp * 16;  // first token of this warp's slice
  if (slice >= len) return;
  if (slice + 16 > len) {
    // Ragged end: zero this warp's V rows at or past the valid length so that whatever the
    // cache holds there (stale values, NaN) never meets a zero weight.
    for (int e = lane; e < 16 * 8 * kBoxes; e += 32) {
      const int r = e / (8 * kBoxes);
      const int rest = e % (8 * kBoxes);
      const int bx = rest / 8, ch = rest % 8;
      if (slice + r >= len)
        *reinterpret_cast<uint4*>(vt + bx * kTile * 128 + (warp * 16 + r) * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
    }
    fence_proxy_async_smem();
    __syncwarp();
  }
  // ---- S^T = K * Q^T for this warp's 16 tokens ----
  float sc[4] = {0.f, 0.f, 0.f, 0.f};
  const uint32_t krow = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
  for (int kk = 0; kk < kKSteps; ++kk) {
    const int chunk = (kk & 3) * 2 + (lane >> 4);
    const uint32_t addr = smem_u32(kt + (kk >> 2) * kTile * 128) + sw128(krow, chunk);
    uint32_t a0, a1, a2, a3;
    ldmatrix_x4(addr, a0, a1, a2, a3);
    mma_bf16_16816(sc, a0, a1, a2, a3, a.qb[kk][0], a.qb[kk][1]);
  }
  // ---- online softmax over tokens (rows g, g+8), heads (2c, 2c+1) ----
  const int tok0 = slice + g, tok1 = slice + g + 8;
  float s0 = tok0 < len ? sc[0] * sl2 : -INFINITY;
  float s1 = tok0 < len ? sc[1] * sl2 : -INFINITY;
  float s2 = tok1 < len ? sc[2] * sl2 : -INFINITY;
  float s3 = tok1 < len ? sc[3] * sl2 : -INFINITY;
  float mx0 = fmaxf(s0, s2), mx1 = fmaxf(s1, s3);
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
  }
  const float n0 = fmaxf(a.m0, mx0), n1 = fmaxf(a.m1, mx1);
  const float pv0 = n0 == -INFINITY ? 0.f : n0;  // never form -inf - -inf
  const float pv1 = n1 == -INFINITY ? 0.f : n1;
  const float corr0 = exp2f(a.m0 - pv0), corr1 = exp2f(a.m1 - pv1);
  const float p0 = exp2f(s0 - pv0), p1 = exp2f(s1 - pv1);
  const float p2 = exp2f(s2 - pv0), p3 = exp2f(s3 - pv1);
  a.l0 = a.l0 * corr0 + (p0 + p2);
  a.l1 = a.l1 * corr1 + (p1 + p3);
  a.m0 = n0;
  a.m1 = n1;
#pragma unroll
  for (int i = 0; i < kKSteps; ++i) {
    a.o[i][0] *= corr0;
    a.o[i][1] *= corr1;
    a.o[i][2] *= corr0;
    a.o[i][3] *= corr1;
  }
  // P^T fragments (bf16, as the reference's P cast) -> B operand of the PV product.
  const uint32_t pb0 = movmatrix_trans(pack_bf16x2(p0, p1));
  const uint32_t pb1 = movmatrix_trans(pack_bf16x2(p2, p3));
  // ---- O^T += V^T * P^T ----
  const uint32_t vrow = warp * 16 + (lane & 7) + ((lane >> 4) & 1) * 8;
#pragma unroll
  for (int i = 0; i < kKSteps; ++i) {
    const int cg = 2 * i + ((lane >> 3) & 1);
    const uint32_t addr = smem_u32(vt + (cg >> 3) * kTile * 128) + sw128(vrow, cg & 7);
    uint32_t a0, a1, a2, a3;
    ldmatrix_x4_trans(addr, a0, a1, a2, a3);
    mma_bf16_16816(a.o[i], a0, a1, a2, a3, pb0, pb1);
  }
}

// Parks this warp's state in shared memory for the cross-warp reduction: per-head (max,
// denominator) pairs in red_ml[warp][head] and O^T columns in red_o[warp][d][head].
template <int D>
__device__ __forceinline__ void park_warp(WarpAcc<D>& a, float* red_o, float* red_ml, int warp, int lane, int G) {
  const int g = lane >> 2, c = lane & 3;
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    a.l0 += __shfl_xor_sync(0xffffffffu, a.l0, off);
    a.l1 += __shfl_xor_sync(0xffffffffu, a.l1, off);
  }
  if (g == 0) {
    red_ml[(warp * kHeadsPad + 2 * c) * 2 + 0] = a.m0;
    red_ml[(warp * kHeadsPad + 2 * c) * 2 + 1] = a.l0;
    red_ml[(warp * kHeadsPad + 2 * c + 1) * 2 + 0] = a.m1;
    red_ml[(warp * kHeadsPad + 2 * c + 1) * 2 + 1] = a.l1;
  }
  if (2 * c < G) {
#pragma unroll
    for (int i = 0; i < D / 16; ++i) {
      float* r0 = red_o + ((warp * D) + 16 * i + g) * kHeadsPad + 2 * c;
      float* r1 = red_o + ((warp * D) + 16 * i + g + 8) * kHeadsPad + 2 * c;
      r0[0] = a.o[i][0];
      r0[1] = a.o[i][1];
      r1[0] = a.o[i][2];
      r1[1] = a.o[i][3];
    }
  }
}

// The CTA's combined state for element e = (head gq, dim d) from the parked warp states:
// M = max_w m_w, L = sum_w l_w 2^(m_w - M), O = sum_w o_w 2^(m_w - M), warps in order.
template <int D>
__device__ __forceinline__ void combine_warps(const float* red_o, const float* red_ml, int gq, int d, float& M,
                                              float& L, float& O) {
  float mw[kConsumerWarps];
  M = -INFINITY;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) {
    mw[w] = red_ml[(w * kHeadsPad + gq) * 2];
    M = fmaxf(M, mw[w]);
  }
  const float piv = M == -INFINITY ? 0.f : M;
  L = 0.f;
  O = 0.f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) {
    const float f = exp2f(mw[w] - piv);
    L += red_ml[(w * kHeadsPad + gq) * 2 + 1] * f;
    O += red_o[((w * D) + d) * kHeadsPad + gq] * f;
  }
}

template <int D, int NS>
struct Smem {
  static constexpr int kBoxes = D / 64;
  static constexpr int kTileBytes = kBoxes * kTile * 128;  // one of K or V
  static constexpr int kStageBytes = 2 * kTileBytes;
  // [stages][K | V] tiles, 1024-byte aligned (swizzle atom)
  static constexpr int kStagesBytes = NS * kStageBytes;
  static constexpr int kRedO = kConsumerWarps * D * kHeadsPad * 4;  // O^T partials per warp
  static constexpr int kRedML = kConsumerWarps * kHeadsPad * 2 * 4;
  static constexpr int kCum = ((kMaxBatch + 1) * 4 + 15) & ~15;  // keeps the mbarriers 8-byte aligned
  static constexpr int kBars = 2 * NS * 8;
  static constexpr int kMisc = 64;
  static constexpr int kMerge = kMaxCtas * kHeadsPad * 4 + kHeadsPad * 4;  // run weights + denominators
  static constexpr int kTotal = 1024 + kStagesBytes + kRedO + kRedML + kCum + kBars + kMisc + kMerge;
  static_assert((kStagesBytes + kRedO + kRedML + kCum) % 16 == 0, "mbarrier alignment");
};

template <int D, int NS>
__global__ void __launch_bounds__(kThreads, 1)
    decode_partials_kernel(const __grid_constant__ CUtensorMap kmap,
                           const __grid_constant__ CUtensorMap vmap, const Params p) {
  using S = Smem<D, NS>;
  constexpr int kBoxes = S::kBoxes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* stages = base;
  float* red_o = reinterpret_cast<float*>(base + S::kStagesBytes);
  float* red_ml = reinterpret_cast<float*>(base + S::kStagesBytes + S::kRedO);
  int* cum = reinterpret_cast<int*>(base + S::kStagesBytes + S::kRedO + S::kRedML);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + S::kStagesBytes + S::kRedO + S::kRedML +
                                               S::kCum);
  uint64_t* empty = full + NS;
  int* misc = reinterpret_cast<int*>(empty + NS);  // [0..2] start b,h,j; [4] abort; [5..7] merge
  float* merge_w = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(misc) + S::kMisc);
  float* merge_den = merge_w + kMaxCtas * kHeadsPad;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int B = p.batch, Hkv = p.kv_heads, G = p.groups;

  // ---- plan: per-row tile prefix sums, this CTA's tile slice and its first tile ----
  if (warp == 0) {
    int running = 0;
    if (lane == 0) cum[0] = 0;
    for (int b0 = 0; b0 < B; b0 += 32) {
      int b = b0 + lane;
      int n = b < B ? tiles_of(row_length(p.position, p.per_row, b, p.capacity)) : 0;
      int x = n;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (b < B) cum[b + 1] = running + x;
      running += __shfl_sync(0xffffffffu, x, 31);
    }
  }
  if (warp == kConsumerWarps && lane == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_barrier_init();
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    misc[4] = 0;
  }
  __syncthreads();

  if (p.counters != nullptr && blockIdx.x == 0) {
    pdl_wait();  // `out` may still be read by an earlier kernel
    // Rows with no valid slot get no run; the fused form writes their (empty) output.
    for (int b = 0; b < B; ++b)
      if (cum[b + 1] == cum[b])
        for (int e = threadIdx.x; e < p.q_heads * (int)D; e += blockDim.x)
          p.out[static_cast<size_t>(b) * p.q_heads * D + e] = __float2bfloat16_rn(0.f);
  }
  const long long total = static_cast<long long>(Hkv) * cum[B];
  const long long t0 = total > 0 ? slice_start(total, blockIdx.x, p.ctas) : 0;
  const long long t1 = total > 0 ? slice_start(total, blockIdx.x + 1, p.ctas) : 0;
  const int count = static_cast<int>(t1 - t0);
  if (count <= 0) return;

  if (warp == 0) {
    for (int b0 = 0; b0 < B; b0 += 32) {
      int b = b0 + lane;
      bool hit = false;
      if (b < B) {
        long long lo = static_cast<long long>(Hkv) * cum[b];
        long long hi = static_cast<long long>(Hkv) * cum[b + 1];
        hit = lo <= t0 && t0 < hi;
      }
      unsigned m = __ballot_sync(0xffffffffu, hit);
      if (m != 0) {
        if (lane == __ffs(m) - 1) {
          int n = cum[b + 1] - cum[b];
          long long off = t0 - static_cast<long long>(Hkv) * cum[b];
          misc[0] = b;
          misc[1] = static_cast<int>(off / n);
          misc[2] = static_cast<int>(off % n);
        }
        break;
      }
    }
  }
  __syncthreads();

  volatile int* abort_flag = &misc[4];

  if (warp == kConsumerWarps) {
    // ===================== producer: one lane issues every TMA =====================
    if (lane == 0) {
      int b = misc[0], h = misc[1], j = misc[2];
      int n = cum[b + 1] - cum[b];
      // Cache rows below a row's position were written by earlier steps, so the ring is
      // filled before the dependency wait; the tile holding the row's newest slot (the
      // previous kernel appends it) waits for the previous kernel.
      bool waited = false;
      for (int k = 0; k < count; ++k) {
        const int s = k % NS;
        if (!waited && (k >= NS || j == n - 1)) {
          pdl_wait();
          waited = true;
        }
        if (*abort_flag) break;
        if (k >= NS) {
          if (!mbar_wait_bounded(&empty[s], ((k / NS) - 1) & 1)) {
            raise_error(p.err, kErrTimeoutEmpty);
            *abort_flag = 1;
            break;
          }
        }
        uint8_t* kt = stages + s * S::kStageBytes;
        uint8_t* vt = kt + S::kTileBytes;
        const int row = (b * Hkv + h) * p.capacity + j * kTile;
        mbar_arrive_expect_tx(&full[s], S::kStageBytes);
#pragma unroll
        for (int bx = 0; bx < kBoxes; ++bx) {
          tma_load_2d(kt + bx * kTile * 128, &kmap, &full[s], bx * 64, row);
          tma_load_2d(vt + bx * kTile * 128, &vmap, &full[s], bx * 64, row);
        }
        if (++j == n) {
          j = 0;
          if (++h == Hkv) {
            h = 0;
            do {
              ++b;
            } while (b < B && cum[b + 1] == cum[b]);
            if (b < B) n = cum[b + 1] - cum[b];
          }
        }
      }
    }
    return;
  }

  // ========================== consumers: warps 0..3 ==========================
  pdl_wait();  // the query rows come from the previous kernel
  pdl_trigger();
  const int ctid = threadIdx.x;  // 0..127

  int b = misc[0], h = misc[1], j = misc[2];
  int n = cum[b + 1] - cum[b];
  int len = row_length(p.position, p.per_row, b, p.capacity);
  int run_first = j;

  WarpAcc<D> acc;
  start_pair<D>(acc, p, b, h, lane);

  const float sl2 = p.scale_log2;
  bool aborted = false;

  for (int k = 0; k < count; ++k) {
    const int s = k % NS;
    if (!mbar_wait_bounded(&full[s], (k / NS) & 1)) {
      raise_error(p.err, kErrTimeoutFull);
      *abort_flag = 1;
      aborted = true;
    }
    if (aborted || *abort_flag) {
      aborted = true;
      break;
    }
    uint8_t* kt = stages + s * S::kStageBytes;
    attend_tile<D>(acc, kt, kt + S::kTileBytes, j * kTile, len, warp, lane, sl2);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    // ---- advance; finalize the run when the pair changes or the slice ends ----
    const int cur_b = b, cur_h = h, cur_first = run_first, cur_last = j, cur_n = n;
    bool run_end = (k == count - 1);
    if (++j == n) {
      j = 0;
      run_end = true;
      if (++h == Hkv) {
        h = 0;
        do {
          ++b;
        } while (b < B && cum[b + 1] == cum[b]);
      }
    }
    if (run_end) {
      park_warp<D>(acc, red_o, red_ml, warp, lane, G);
      asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
      const bool whole = cur_first == 0 && cur_last == cur_n - 1;
      const int pair = cur_b * Hkv + cur_h;
      const int slot = blockIdx.x + pair;
      for (int e = ctid; e < G * D; e += kConsumerWarps * 32) {
        const int gq = e / D, d = e % D;
        float M, L, O;
        combine_warps<D>(red_o, red_ml, gq, d, M, L, O);
        if (whole) {
          p.out[(static_cast<size_t>(cur_b) * p.q_heads + cur_h * G + gq) * D + d] =
              __float2bfloat16_rn(O / L);
        } else {
          p.acc[(static_cast<size_t>(slot) * G + gq) * D + d] = O;
          if (d == 0) p.stats[static_cast<size_t>(slot) * G + gq] = make_float2(M, L);
        }
      }
      if (!whole && p.counters != nullptr) {
        // Publish this run, count it, and let the pair's last run merge them all.
        __threadfence();
        asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
        if (ctid == 0) {
          const long long first = static_cast<long long>(Hkv) * cum[cur_b] + static_cast<long long>(cur_h) * cur_n;
          const int lo = slice_owner(total, first, p.ctas);
          const int hi = slice_owner(total, first + cur_n - 1, p.ctas);
          int runs = hi - lo + 1;
          if (total < p.ctas) {  // some slices are empty: count the CTAs that really ran
            runs = 0;
            for (int i = lo; i <= hi; ++i)
              runs += slice_start(total, i, p.ctas) < slice_start(total, i + 1, p.ctas);
          }
          const int done = atomicAdd(&p.counters[pair], 1);
          const int last = done == runs - 1;
          if (last) p.counters[pair] = 0;  // every run of this launch has counted: reset for the next
          misc[5] = last;
          misc[6] = lo;
          misc[7] = hi;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
        if (misc[5]) {
          __threadfence();
          merge_pair<D, kConsumerWarps * 32>(p, pair, misc[6], misc[7], total, ctid, merge_w, merge_den,
                                              [] { asm volatile("bar.sync 1, 128;" ::: "memory"); });
        }
      }
      asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
      if (k != count - 1) {
        n = cum[b + 1] - cum[b];
        len = row_length(p.position, p.per_row, b, p.capacity);
        run_first = j;
        start_pair<D>(acc, p, b, h, lane);
      }
    }
  }
  if (aborted) {
    // Let copies already issued land before the CTA's shared memory is released.
    __syncwarp();
  }
}

// One CTA per (row, KV head): merge the runs of the CTAs that shared the pair. The
// contributing CTAs and their per-head softmax weights exp2(m_run - M) are resolved once
// into shared memory; the weighted sum over runs is then a coalesced sweep over the
// partial accumulators, in increasing CTA order (deterministic).
constexpr int kCombineThreads = 256;

template <int D>
__global__ void __launch_bounds__(kCombineThreads, 1) decode_combine_kernel(const Params p) {
  __shared__ int s_before, s_total, s_n;
  __shared__ float s_w[kMaxCtas * kHeadsPad];
  __shared__ float s_den[kHeadsPad];
  pdl_wait();
  pdl_trigger();
  const int pair = blockIdx.x;
  const int b = pair / p.kv_heads, h = pair % p.kv_heads;
  const int G = p.groups;
  if (threadIdx.x == 0) {
    s_before = 0;
    s_total = 0;
    s_n = 0;
  }
  __syncthreads();
  int before = 0, total = 0;
  for (int r = threadIdx.x; r < p.batch; r += blockDim.x) {
    const int n = tiles_of(row_length(p.position, p.per_row, r, p.capacity));
    total += n;
    if (r < b) before += n;
    if (r == b) s_n = n;
  }
  if (before) atomicAdd(&s_before, before);
  if (total) atomicAdd(&s_total, total);
  __syncthreads();
  const int n = s_n;
  const long long T = static_cast<long long>(p.kv_heads) * s_total;
  if (n == 0) {
    __nv_bfloat16* out = p.out + (static_cast<size_t>(b) * p.q_heads + h * G) * D;
    for (int e = threadIdx.x; e < G * D; e += blockDim.x) out[e] = __float2bfloat16_rn(0.f);
    return;
  }
  const long long first = static_cast<long long>(p.kv_heads) * s_before + static_cast<long long>(h) * n;
  const int lo = slice_owner(T, first, p.ctas);
  const int hi = slice_owner(T, first + n - 1, p.ctas);
  if (lo == hi) return;  // one run covered the pair and wrote the output itself
  merge_pair<D, kCombineThreads>(p, pair, lo, hi, T, threadIdx.x, s_w, s_den, [] { __syncthreads(); });
}


// ---------------------------------------------------------------------------------------
// Cluster form, for a position shared by every row and few (row, KV head) pairs (tensor-
// parallel shards, small batches): one thread-block cluster of C <= 16 CTAs per pair. CTA r
// streams tiles r, r + C, r + 2C, ... of the pair (interleaved: measured ~3% faster than
// contiguous slices on B200) with the same per-tile arithmetic as the persistent kernel. CTA r owns outputs [r*chunk, (r+1)*chunk) of the pair's G*D values: every
// CTA stores its partial O of each output into the owner's shared memory, and its per-head
// (max, denominator) into every CTA's, with remote (DSMEM) stores; after one cluster barrier
// each CTA merges its outputs over the C partials from its own shared memory, in rank order.
// No global partials, fences, counters, second pass, or remote loads on the critical path.
// ---------------------------------------------------------------------------------------
constexpr int kMaxCluster = 16;  // 16 needs the non-portable cluster size attribute

template <int D, int NS>
struct ClusterSmem {
  static constexpr int kBoxes = D / 64;
  static constexpr int kTileBytes = kBoxes * kTile * 128;
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kStagesBytes = NS * kStageBytes;
  // the warps' O^T partials reuse the drained stage ring
  static constexpr int kRedO = kConsumerWarps * D * kHeadsPad * 4;
  static_assert(kRedO <= kStagesBytes, "the warp partials must fit the stage ring");
  static constexpr int kRedML = kConsumerWarps * kHeadsPad * 2 * 4;
  // partials received as an owner: O of [rank][chunk] (C * ceil(G*D / C) <= G*D + C - 1 values)
  // and every rank's (max, denominator) per head
  static constexpr int kRecvO = ((kHeadsPad * D + kMaxCluster) * 4 + 15) / 16 * 16;
  static constexpr int kRecvML = kMaxCluster * kHeadsPad * 2 * 4;
  static constexpr int kBars = 2 * NS * 8;
  static constexpr int kTotal = 1024 + kStagesBytes + kRedML + kRecvO + kRecvML + kBars + 16;
  static_assert((kStagesBytes + kRedML + kRecvO + kRecvML) % 16 == 0, "mbarrier alignment");
};

template <int D, int NS>
__global__ void __launch_bounds__(kThreads, 1)
    decode_cluster_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                          const Params p) {
  using S = ClusterSmem<D, NS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = base;
  float* red_o = reinterpret_cast<float*>(base);  // used once the ring has drained
  float* red_ml = reinterpret_cast<float*>(base + S::kStagesBytes);
  float* recv_o = red_ml + S::kRedML / 4;    // [sender rank][chunk]
  float* recv_ml = recv_o + S::kRecvO / 4;   // [sender rank][head][max, denominator]
  uint64_t* full = reinterpret_cast<uint64_t*>(recv_ml + S::kRecvML / 4);
  uint64_t* empty = full + NS;
  int* abort_word = reinterpret_cast<int*>(empty + NS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = gridDim.x;
  const int rank = blockIdx.x;  // cluster dims (C, 1, 1): the CTA's rank in its cluster
  const int pair = blockIdx.y;
  const int Hkv = p.kv_heads, G = p.groups;
  const int b = pair / Hkv, h = pair % Hkv;
  // the shared position was written before this step: read before the dependency wait
  const int len = row_length(p.position, 0, b, p.capacity);
  const int n = tiles_of(len);
  const int count = n > rank ? (n - rank + C - 1) / C : 0;  // tiles rank, rank + C, ...

  // Every thread announces that its CTA runs; the wait before the first remote store then
  // costs nothing (a CTA's shared memory may only be written once its CTA has started).
  cluster_arrive_relaxed();
  if (warp == kConsumerWarps && lane == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_barrier_init();
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    *abort_word = 0;
  }
  __syncthreads();
  volatile int* abort_flag = abort_word;

  if (warp == kConsumerWarps) {
    // ===================== producer: one lane issues every TMA =====================
    if (lane == 0) {
      // Cache rows below the position were written by earlier steps: the ring is filled
      // before the dependency wait; the row's last tile (the previous kernel appends its
      // newest slot) waits for the previous kernel.
      bool waited = false;
      for (int k = 0; k < count; ++k) {
        const int s = k % NS;
        const int j = rank + k * C;
        if (!waited && (k >= NS || j == n - 1)) {
          pdl_wait();
          waited = true;
        }
        if (*abort_flag) break;
        if (k >= NS && !mbar_wait_bounded(&empty[s], ((k / NS) - 1) & 1)) {
          raise_error(p.err, kErrTimeoutEmpty);
          *abort_flag = 1;
          break;
        }
        uint8_t* kt = stages + s * S::kStageBytes;
        uint8_t* vt = kt + S::kTileBytes;
        const int row = (b * Hkv + h) * p.capacity + j * kTile;
        mbar_arrive_expect_tx(&full[s], S::kStageBytes);
#pragma unroll
        for (int bx = 0; bx < S::kBoxes; ++bx) {
          tma_load_2d(kt + bx * kTile * 128, &kmap, &full[s], bx * 64, row);
          tma_load_2d(vt + bx * kTile * 128, &vmap, &full[s], bx * 64, row);
        }
      }
    }
    __syncwarp();
    // every thread of every CTA in the cluster completes the same two barrier phases
    cluster_wait();
    cluster_sync();
    return;
  }

  // ========================== consumers: warps 0..3 ==========================
  pdl_wait();  // the query rows come from the previous kernel
  pdl_trigger();
  const int ctid = threadIdx.x;  // 0..127
  WarpAcc<D> acc;
  start_pair<D>(acc, p, b, h, lane);
  bool aborted = false;
  for (int k = 0; k < count; ++k) {
    const int s = k % NS;
    if (!mbar_wait_bounded(&full[s], (k / NS) & 1)) {
      raise_error(p.err, kErrTimeoutFull);
      *abort_flag = 1;
      aborted = true;
    }
    if (aborted || *abort_flag) {
      aborted = true;  // still takes the cluster barriers below
      break;
    }
    uint8_t* kt = stages + s * S::kStageBytes;
    attend_tile<D>(acc, kt, kt + S::kTileBytes, (rank + k * C) * kTile, len, warp, lane, p.scale_log2);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  // this CTA's partial: (M, L) per head, O per (head, dim); an empty slice gives (-inf, 0, 0).
  // Every warp is done with the stage ring (red_o overlays it) and no copy is in flight: the
  // producer issued exactly `count` tiles and each was consumed, or the loop aborted.
  asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
  park_warp<D>(acc, red_o, red_ml, warp, lane, G);
  asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
  const int total = G * D, chunk = (total + C - 1) / C;
  cluster_wait();  // every CTA of the cluster runs: its shared memory may be written
  for (int e = ctid; e < total; e += kConsumerWarps * 32) {
    const int gq = e / D, d = e % D;
    float M, L, O;
    combine_warps<D>(red_o, red_ml, gq, d, M, L, O);
    const int owner = e / chunk;
    st_cluster_f32(map_shared(smem_u32(&recv_o[rank * chunk + (e - owner * chunk)]), owner), O);
    if (d == 0) {
      for (int q = 0; q < C; ++q) {
        st_cluster_f32(map_shared(smem_u32(&recv_ml[(rank * kHeadsPad + gq) * 2]), q), M);
        st_cluster_f32(map_shared(smem_u32(&recv_ml[(rank * kHeadsPad + gq) * 2 + 1]), q), L);
      }
    }
  }
  cluster_sync();  // every partial has landed; no CTA touches another's shared memory after this
  // this CTA's outputs, summed over the cluster in rank order
  const int e0 = rank * chunk, e1 = min(total, e0 + chunk);
  __nv_bfloat16* out = p.out + (static_cast<size_t>(b) * p.q_heads + h * G) * D;
  for (int e = e0 + ctid; e < e1; e += kConsumerWarps * 32) {
    const int gq = e / D;
    float mq[kMaxCluster];
    float M = -INFINITY;
#pragma unroll
    for (int q = 0; q < kMaxCluster; ++q)
      if (q < C) {
        mq[q] = recv_ml[(q * kHeadsPad + gq) * 2];
        M = fmaxf(M, mq[q]);
      }
    const float piv = M == -INFINITY ? 0.f : M;
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int q = 0; q < kMaxCluster; ++q)
      if (q < C) {
        const float w = exp2f(mq[q] - piv);
        L += recv_ml[(q * kHeadsPad + gq) * 2 + 1] * w;
        O += recv_o[q * chunk + (e - e0)] * w;
      }
    out[e] = __float2bfloat16_rn(L > 0.f ? O / L : 0.f);  // a row with no valid slot writes zeros
  }
}

constexpr int kStages = 4;
constexpr int kClusterStages = 2;  // the cluster form's small ring: three CTAs per SM

template <int D, int NS>
bool configure_cluster() {
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(decode_cluster_kernel<D, NS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             ClusterSmem<D, NS>::kTotal) != cudaSuccess)
      return false;
    if (cudaFuncSetAttribute(decode_cluster_kernel<D, NS>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) !=
        cudaSuccess)
      cudaGetLastError();  // no clusters above 8: the occupancy query then reports none
    configured[dev] = true;
  }
  return true;
}

// Clusters of `c` CTAs of the cluster kernel that the device holds at once (-1 if unknown),
// cached per (device, head dim, stages, c).
template <int D, int NS>
int resident_clusters(int c) {
  static int cache[64][kMaxCluster + 1] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && cache[dev][c] != 0) return cache[dev][c];
  if (!configure_cluster<D, NS>()) return -1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(c, 1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = ClusterSmem<D, NS>::kTotal;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = c;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, decode_cluster_kernel<D, NS>, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = -1;  // unknown: never chosen
  }
  if (dev < 64) cache[dev][c] = n;
  return n;
}

// The largest cluster size in [2, limit] whose `pairs` clusters are all resident at once, or 0.
// Any size counts, not only powers of two: 16 pairs fill 144 SMs with clusters of 9.
template <int D, int NS>
int cluster_size(int pairs, int limit) {
  for (int c = limit; c >= 2; --c)
    if (resident_clusters<D, NS>(c) >= pairs) return c;
  return 0;
}

template <int D, int NS>
int launch_cluster(const CUtensorMap& km, const CUtensorMap& vm, const Params& p, int cluster, cudaStream_t stream) {
  if (!configure_cluster<D, NS>()) return FB_ERR_LAUNCH;
  return launch_ex(decode_cluster_kernel<D, NS>, dim3(cluster, p.batch * p.kv_heads), dim3(kThreads),
                   ClusterSmem<D, NS>::kTotal, stream, cluster, km, vm, p);
}

// Tuning override of the cluster form's shape (fb_decode_attention_cluster_shape): cluster
// size and ring depth, 0 = automatic.
int g_force_cluster = 0, g_force_stages = 0;

template <int D>
int launch_cluster_stages(const CUtensorMap& km, const CUtensorMap& vm, const Params& p, int c, int ns,
                          cudaStream_t s) {
  if (ns == 2) return launch_cluster<D, 2>(km, vm, p, c, s);
  if (ns == 3) return launch_cluster<D, 3>(km, vm, p, c, s);
  return launch_cluster<D, kStages>(km, vm, p, c, s);
}

template <int D>
int resident_clusters_stages(int c, int ns) {
  if (ns == 2) return resident_clusters<D, 2>(c);
  if (ns == 3) return resident_clusters<D, 3>(c);
  return resident_clusters<D, kStages>(c);
}

// Cluster form choice (measured on B200, 16 rows x 8193 tokens, graph-timed, power-of-two
// sizes): the 4-stage ring (one CTA per SM) while its clusters cover about two thirds of the
// SMs or more (64 pairs: 2 x 64 CTAs, 45.9 us against 46.4-51.2 for 4x2, 4x3, 8x2; 32 pairs: 4 x
// 32, 25.2 us against 25.7-31.0 for 8x3, 4x3, 8x2, 16x2); below that the larger clusters of the
// 3-stage ring (two CTAs per SM) or the 2-stage ring (three) (16 pairs: 8 x 16 CTAs with 3
// stages 17.1 us, 2 stages 18.6, 16 x 16 with 2 stages 17.2, 4 x 16 with 4 stages 20.4). The
// 4-stage ring takes the largest cluster that keeps one CTA per SM (16 pairs: 9 x 16 = 144
// CTAs). Returns FB_ERR_SHAPE when none fits in one wave.
template <int D>
int launch_cluster_form(const CUtensorMap& km, const CUtensorMap& vm, const Params& p, int pairs, cudaStream_t s) {
  if (g_force_cluster >= 2) {
    const int ns = g_force_stages;
    if (resident_clusters_stages<D>(g_force_cluster, ns) < pairs) return FB_ERR_SHAPE;
    return launch_cluster_stages<D>(km, vm, p, g_force_cluster, ns, s);
  }
  const int one_per_sm = sm_count() / pairs < kMaxCluster ? sm_count() / pairs : kMaxCluster;
  const int c4 = cluster_size<D, kStages>(pairs, one_per_sm);
  if (c4 >= 2 && 3 * pairs * c4 >= 2 * sm_count()) return launch_cluster<D, kStages>(km, vm, p, c4, s);
  // clusters of 16 (non-portable) only when clusters of 8 would leave half the SMs idle
  const int limit = 2 * pairs * 8 <= sm_count() ? kMaxCluster : 8;
  const int c3 = cluster_size<D, 3>(pairs, limit);
  const int c2 = cluster_size<D, kClusterStages>(pairs, limit);
  if (c3 > c4 && c3 >= c2) return launch_cluster<D, 3>(km, vm, p, c3, s);
  if (c2 > c4) return launch_cluster<D, kClusterStages>(km, vm, p, c2, s);
  if (c4 >= 2) return launch_cluster<D, kStages>(km, vm, p, c4, s);
  return FB_ERR_SHAPE;
}

template <int D>
int launch_partials(const CUtensorMap& km, const CUtensorMap& vm, const Params& p,
                    cudaStream_t stream) {
  using S = Smem<D, kStages>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(decode_partials_kernel<D, kStages>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal) != cudaSuccess)
      return FB_ERR_LAUNCH;
    configured[dev] = true;
  }
  return launch_ex(decode_partials_kernel<D, kStages>, dim3(p.ctas), dim3(kThreads), S::kTotal, stream, 1, km, vm,
                   p);
}

int validate(int batch, int q_heads, int kv_heads, int head_dim, int capacity) {
  if (batch <= 0 || q_heads <= 0 || kv_heads <= 0 || capacity <= 0) return FB_ERR_ARG;
  if (head_dim != 64 && head_dim != 128) return FB_ERR_SHAPE;
  if (q_heads % kv_heads != 0 || q_heads / kv_heads > kHeadsPad) return FB_ERR_SHAPE;
  if (batch > kMaxBatch) return FB_ERR_SHAPE;
  if (static_cast<long long>(batch) * kv_heads * capacity >= (1ll << 31)) return FB_ERR_SHAPE;
  return FB_OK;
}

}  // namespace attn
}  // namespace fb

using namespace fb;
using namespace fb::attn;

extern "C" int fb_decode_attention_ctas(int batch, int kv_heads, int capacity, int head_dim) {
  (void)batch;
  (void)kv_heads;
  (void)capacity;
  (void)head_dim;
  return sm_count();
}

extern "C" int fb_decode_attention_cluster_shape(int cluster, int stages) {
  if (cluster == 0) {
    g_force_cluster = g_force_stages = 0;
    return FB_OK;
  }
  if (cluster < 2 || cluster > kMaxCluster || stages < 2 || stages > kStages) return FB_ERR_ARG;
  g_force_cluster = cluster;
  g_force_stages = stages;
  return FB_OK;
}

extern "C" size_t fb_decode_attention_workspace(int batch, int q_heads, int kv_heads,
                                                int head_dim, int ctas) {
  if (batch <= 0 || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || ctas <= 0) return 0;
  const size_t G = q_heads / kv_heads;
  const size_t slots = static_cast<size_t>(ctas) + static_cast<size_t>(batch) * kv_heads;
  const size_t acc = ((slots * G * head_dim * sizeof(float)) + 255) & ~size_t(255);
  const size_t stats = ((slots * G * sizeof(float2)) + 255) & ~size_t(255);
  const size_t counters = static_cast<size_t>(batch) * kv_heads * sizeof(int);
  return acc + stats + counters;
}

static int make_params(Params* p, const void* q, const int64_t* position, int per_row, void* out,
                       void* workspace, size_t workspace_bytes, int batch, int q_heads,
                       int kv_heads, int head_dim, int capacity, float scale, int ctas, bool fused) {
  int st = validate(batch, q_heads, kv_heads, head_dim, capacity);
  if (st != FB_OK) return st;
  if (position == nullptr || out == nullptr || workspace == nullptr || ctas <= 0) return FB_ERR_ARG;
  if (ctas > kMaxCtas) return FB_ERR_SHAPE;
  const size_t need = fb_decode_attention_workspace(batch, q_heads, kv_heads, head_dim, ctas);
  if (workspace_bytes < need) return FB_ERR_WORKSPACE;
  const size_t G = q_heads / kv_heads;
  const size_t slots = static_cast<size_t>(ctas) + static_cast<size_t>(batch) * kv_heads;
  const size_t acc = ((slots * G * head_dim * sizeof(float)) + 255) & ~size_t(255);
  const size_t stats = ((slots * G * sizeof(float2)) + 255) & ~size_t(255);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p->q = static_cast<const __nv_bfloat16*>(q);
  p->position = position;
  p->per_row = per_row ? 1 : 0;
  p->out = static_cast<__nv_bfloat16*>(out);
  p->acc = reinterpret_cast<float*>(ws);
  p->stats = reinterpret_cast<float2*>(ws + acc);
  p->counters = fused ? reinterpret_cast<int*>(ws + acc + stats) : nullptr;
  p->batch = batch;
  p->q_heads = q_heads;
  p->kv_heads = kv_heads;
  p->groups = q_heads / kv_heads;
  p->capacity = capacity;
  p->ctas = ctas;
  p->scale_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634);
  p->err = error_word();
  return FB_OK;
}

static int launch_decode(const void* q, const void* k, const void* v, const int64_t* position,
                         int per_row, void* out, void* workspace, size_t workspace_bytes, int batch,
                         int q_heads, int kv_heads, int head_dim, int capacity, float scale,
                         int ctas, void* stream, bool fused) {
  if (q == nullptr || k == nullptr || v == nullptr) return FB_ERR_ARG;
  Params p;
  int st = make_params(&p, q, position, per_row, out, workspace, workspace_bytes, batch, q_heads,
                       kv_heads, head_dim, capacity, scale, ctas, fused);
  if (st != FB_OK) return st;
  const uint64_t rows = static_cast<uint64_t>(batch) * kv_heads * capacity;
  CUtensorMap km, vm;
  st = encode_bf16_2d(&km, k, rows, head_dim, head_dim, 64, kTile, true);
  if (st != FB_OK) return st;
  st = encode_bf16_2d(&vm, v, rows, head_dim, head_dim, 64, kTile, true);
  if (st != FB_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // A shared position and few pairs: one cluster per pair, merged through DSMEM, when the
  // clusters all fit in one wave.
  const int pairs = batch * kv_heads;
  if (fused && !per_row && 2 * pairs <= sm_count()) {
    st = head_dim == 128 ? launch_cluster_form<128>(km, vm, p, pairs, s) : launch_cluster_form<64>(km, vm, p, pairs, s);
    // a forced shape (fb_decode_attention_cluster_shape) that does not fit one wave is an error
    if (st != FB_ERR_SHAPE || g_force_cluster >= 2) return st;
  }
  return head_dim == 128 ? launch_partials<128>(km, vm, p, s) : launch_partials<64>(km, vm, p, s);
}

extern "C" int fb_decode_attention(const void* q, const void* k, const void* v,
                                   const int64_t* position, int per_row, void* out, void* workspace,
                                   size_t workspace_bytes, int batch, int q_heads, int kv_heads,
                                   int head_dim, int capacity, float scale, int ctas,
                                   void* stream) {
  return launch_decode(q, k, v, position, per_row, out, workspace, workspace_bytes, batch, q_heads,
                       kv_heads, head_dim, capacity, scale, ctas, stream, true);
}

extern "C" int fb_decode_attention_partials(const void* q, const void* k, const void* v,
                                            const int64_t* position, int per_row, void* out,
                                            void* workspace, size_t workspace_bytes, int batch,
                                            int q_heads, int kv_heads, int head_dim, int capacity,
                                            float scale, int ctas, void* stream) {
  return launch_decode(q, k, v, position, per_row, out, workspace, workspace_bytes, batch, q_heads,
                       kv_heads, head_dim, capacity, scale, ctas, stream, false);
}

extern "C" int fb_decode_attention_combine(const int64_t* position, int per_row, void* out,
                                           void* workspace, size_t workspace_bytes, int batch,
                                           int q_heads, int kv_heads, int head_dim, int capacity,
                                           int ctas, void* stream) {
  Params p;
  int st = make_params(&p, nullptr, position, per_row, out, workspace, workspace_bytes, batch,
                       q_heads, kv_heads, head_dim, capacity, 1.0f, ctas, false);
  if (st != FB_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int pairs = batch * kv_heads;
  if (head_dim == 128) return launch_ex(decode_combine_kernel<128>, dim3(pairs), dim3(kCombineThreads), 0, s, 1, p);
  return launch_ex(decode_combine_kernel<64>, dim3(pairs), dim3(kCombineThreads), 0, s, 1, p);
}

// ---------------------------------------------------------------------------------------
// Decode attention whose scratch is a fixed array inside this library, for callers that
// cannot allocate device memory (no counterpart in the reference). Such a caller owns all
// device memory itself - for example a serving runtime with a fixed, pre-reserved pool that
// hands kernels only their input and output buffers, or a plugin host whose allocator must
// not be called from the plugin - so it cannot provide fb_decode_attention's workspace.
// ---------------------------------------------------------------------------------------
namespace fb {
namespace attn {

constexpr int kNoAllocMaxPairs = 512;  // batch * kv_heads
constexpr int kNoAllocMaxCtas = 160;   // persistent CTAs used by this entry point
// Sized for the largest request accepted: (ctas + pairs) run slots of up to 8 heads x 128
// dims of fp32 partials, their (max, sum) stats, and one counter per pair.
constexpr size_t kNoAllocScratchBytes =
    ((static_cast<size_t>(kNoAllocMaxCtas + kNoAllocMaxPairs) * kHeadsPad * 128 * 4 + 255) &
     ~size_t(255)) +
    ((static_cast<size_t>(kNoAllocMaxCtas + kNoAllocMaxPairs) * kHeadsPad * 8 + 255) & ~size_t(255)) +
    static_cast<size_t>(kNoAllocMaxPairs) * 4;

// Every GPU that loads the library holds this array until the process exits. In host code
// the name is only a stand-in: the device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
void* g_noalloc_address[64] = {nullptr};

// Device address of the scratch array on the current device, looked up once per device
// (with that device current). nullptr if the lookup fails.
void* noalloc_scratch() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_address[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) return nullptr;
    g_noalloc_address[dev] = ptr;
  }
  return g_noalloc_address[dev];
}

}  // namespace attn
}  // namespace fb

extern "C" int fb_decode_attention_noalloc(const void* q, const void* k, const void* v,
                                           const int64_t* position, int per_row, void* out,
                                           int batch, int q_heads, int kv_heads, int head_dim,
                                           int capacity, float scale, void* stream) {
  int st = validate(batch, q_heads, kv_heads, head_dim, capacity);
  if (st != FB_OK) return st;
  if (q == nullptr || k == nullptr || v == nullptr || position == nullptr || out == nullptr)
    return FB_ERR_ARG;
  if (static_cast<long long>(batch) * kv_heads > kNoAllocMaxPairs) return FB_ERR_TOO_LARGE;
  int ctas = sm_count();
  if (ctas > kNoAllocMaxCtas) ctas = kNoAllocMaxCtas;
  const size_t need = fb_decode_attention_workspace(batch, q_heads, kv_heads, head_dim, ctas);
  if (need == 0 || need > kNoAllocScratchBytes) return FB_ERR_TOO_LARGE;
  void* scratch = noalloc_scratch();
  if (scratch == nullptr) return FB_ERR_LAUNCH;
  // The per-pair counters (the workspace's tail) must start at zero: clear them here, since
  // the array keeps whatever the previous call left.
  const size_t counters = static_cast<size_t>(batch) * kv_heads * sizeof(int);
  if (cudaMemsetAsync(static_cast<uint8_t*>(scratch) + need - counters, 0, counters,
                      static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return FB_ERR_LAUNCH;
  return launch_decode(q, k, v, position, per_row, out, scratch, need, batch, q_heads, kv_heads,
                       head_dim, capacity, scale, ctas, stream, true);
}

// Speculative-verify (q_len > 1) attention on the 5th-generation tensor cores (sm_100a).
//
// Semantics follow the reference's `_block_partials` / `_block_merge`
// (engine/kernels/decode_attention.py:260-350, :455-478) and its wrapper `block_attention`
// (:637-680): for row b, KV head h and the T block tokens sitting at slots position[b] + t,
// the T*G query rows ("members", member m = t*G + g) share every K/V tile. Token t < chain[b]
// sees slots [0, position[b] + t]; a later token (an alternative first draft) sees
// [0, position[b]] plus its own slot (:286-292, :323). fp32 scores scaled by scale*log2(e),
// exp2 online softmax with a -inf-safe pivot (:327), P rounded to bf16 for the value product,
// and an LSE merge across KV splits.
//
// B200 design:
//  * One CTA per (row, KV head, KV split, 32-member group). A producer warp streams
//    128-token K and V tiles with 2-D TMA (128-byte swizzle, no multicast) into a 2-stage ring.
//  * S^T = K_tile * Q^T is one tcgen05.mma chain (M = 128 tokens, N = 32 members, K = D)
//    with the fp32 accumulator in TMEM. Q sits in shared memory in the same swizzled K-major
//    layout, written once by the CTA.
//  * Four softmax warps each read 32 TMEM lanes (one token per thread, 32 member columns),
//    reduce column maxima with a shuffle transpose-reduce and shared memory, and write P as
//    bf16 into a K-major swizzled tile.
//  * O^T_tile = V^T * P^T is a second tcgen05.mma chain (M = 128 dims, N = 32 members,
//    K = 128 tokens) with V read in place as an MN-major operand; each thread (one dim)
//    folds the tile into its fp32 running output with the softmax correction.
//  * Every mbarrier wait is bounded; TMEM is freed on every path.
#include "common.cuh"

namespace fb {
namespace verify {

constexpr int kTile = 128;          // tokens per K/V tile (UMMA M of the score product)
constexpr int kMembers = 32;        // member columns per CTA (UMMA N)
constexpr int kStages = 2;
constexpr int kSoftmaxWarps = 4;    // 128 threads = 128 TMEM lanes
constexpr int kThreads = (kSoftmaxWarps + 1) * 32;
constexpr int kTmemCols = 64;       // S^T (32 columns) + O^T tile (32 columns)

struct Params {
  const __nv_bfloat16* q;  // [B, T, Hq, D] token-major
  const int64_t* position; // [B]
  const int64_t* chain;    // [B]
  __nv_bfloat16* out;      // [B, T, Hq, D]
  float* acc;              // [pairs, S, members_pad, D] (splits > 1)
  float2* stats;           // [pairs, S, members_pad]
  int batch, tokens, q_heads, kv_heads, groups, capacity, splits, chunk, members_pad;
  float scale_log2;
  unsigned* err;
};

// ---- tcgen05 helpers --------------------------------------------------------------------
__device__ __forceinline__ uint64_t umma_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  // sm_100 shared-memory matrix descriptor: start>>4 [0,14), LBO>>4 [16,30), SBO>>4 [32,46),
  // version 1 [46,48), base offset 0, layout SWIZZLE_128B (2) [61,64).
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// kind::f16 instruction descriptor: bf16 x bf16 -> fp32, M = 128, N = kMembers.
__host__ __device__ constexpr uint32_t idesc_bf16(bool a_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) |
         (static_cast<uint32_t>(kMembers >> 3) << 17) | (static_cast<uint32_t>(kTile >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Column-wise reduction of a 32x32 block held one row per lane: afterwards lane c holds the
// reduction of column c (shuffle transpose-reduce, 31 shuffles).
template <bool kMax>
__device__ __forceinline__ float transpose_reduce(float (&v)[32], int lane) {
  float a[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) a[i] = v[i];
#pragma unroll
  for (int width = 16; width >= 1; width >>= 1) {
    const bool upper = (lane & width) != 0;
#pragma unroll
    for (int i = 0; i < width; ++i) {
      const float mine = upper ? a[width + i] : a[i];
      const float other = upper ? a[i] : a[width + i];
      const float recv = __shfl_xor_sync(0xffffffffu, other, width);
      a[i] = kMax ? fmaxf(mine, recv) : mine + recv;
    }
  }
  return a[0];
}

struct Smem {
  static constexpr int kTileBytes = 2 * kTile * 128;       // one of K or V: two 64-dim boxes
  static constexpr int kStageBytes = 2 * kTileBytes;       // K then V
  static constexpr int kQBytes = 2 * kMembers * 128;       // two 64-dim boxes of 32 rows
  static constexpr int kPBytes = 2 * kMembers * 128;       // two 64-token boxes of 32 rows
  static constexpr int kRed = kSoftmaxWarps * kMembers * 4;
  static constexpr int kCol = 4 * kMembers * 4;            // run max, pivot, correction, mask data
  static constexpr int kBars = (2 * kStages + 2) * 8;
  static constexpr int kTotal = 1024 + kStages * kStageBytes + kQBytes + kPBytes + kRed + kCol + 2 * kMembers * 4 + kBars + 32;
};

__global__ void __launch_bounds__(kThreads, 1)
    verify_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                  const Params p) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = base;
  uint8_t* q_s = base + kStages * Smem::kStageBytes;
  uint8_t* p_s = q_s + Smem::kQBytes;
  float* red = reinterpret_cast<float*>(p_s + Smem::kPBytes);
  float* col_max = red + kSoftmaxWarps * kMembers;   // running max per member
  float* col_piv = col_max + kMembers;
  float* col_corr = col_piv + kMembers;
  int* col_valid = reinterpret_cast<int*>(col_corr + kMembers);
  int* col_own = col_valid + kMembers;
  uint64_t* full = reinterpret_cast<uint64_t*>(col_own + kMembers);
  uint64_t* empty = full + kStages;
  uint64_t* mma_bar = empty + kStages;  // [0] scores done, [1] values done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int pair = blockIdx.x, split = blockIdx.y, group0 = blockIdx.z * kMembers;
  const int b = pair / p.kv_heads, h = pair % p.kv_heads;
  const int G = p.groups, T = p.tokens, members = T * G;
  const long long first = p.position[b] + 1;             // first block token's slot + 1
  long long end = first + T - 1;                          // one past the last block slot
  if (end > p.capacity) end = p.capacity;
  const long long begin = static_cast<long long>(split) * p.chunk;
  long long stop = begin + p.chunk;
  if (stop > end) stop = end;
  const int tiles = stop > begin ? static_cast<int>((stop - begin + kTile - 1) / kTile) : 0;

  // ---- set-up: barriers, TMEM, Q tile, per-member visibility ----
  if (warp == kSoftmaxWarps && lane == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&mma_bar[0], 1);
    mbar_init(&mma_bar[1], 1);
    fence_barrier_init();
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    *abort_flag = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  // Q members [group0, group0 + 32) of this (row, KV head) into the swizzled K-major tile;
  // rows past the real members are zero.
  for (int e = tid; e < kMembers * 16; e += blockDim.x) {
    const int r = e / 16, c16 = e % 16;  // member row, 16-byte chunk of D = 128
    const int m = group0 + r;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (m < members) {
      const int t = m / G, g = m % G;
      const __nv_bfloat16* src =
          p.q + ((static_cast<size_t>(b) * T + t) * p.q_heads + h * G + g) * 128 + c16 * 8;
      v = *reinterpret_cast<const uint4*>(src);
    }
    *reinterpret_cast<uint4*>(q_s + (c16 >> 3) * (kMembers * 128) + sw128(r, c16 & 7)) = v;
  }
  if (tid < kMembers) {
    const int m = group0 + tid;
    const int t = m / G;
    const bool live = m < members;
    const bool chained = live && t < p.chain[b];
    col_valid[tid] = live ? static_cast<int>(first + (chained ? t : 0)) : 0;
    col_own[tid] = live && !chained ? static_cast<int>(first - 1 + t) : -1;
    col_max[tid] = -INFINITY;
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_s = tmem;              // columns [0, 32): S^T
  const uint32_t tmem_o = tmem + kMembers;   // columns [32, 64): O^T of the current tile

  if (warp == kSoftmaxWarps) {
    // ============================ TMA producer ============================
    if (lane == 0) {
      const int row0 = pair * p.capacity + static_cast<int>(begin);
      for (int i = 0; i < tiles && !*abort_flag; ++i) {
        const int s = i % kStages;
        if (i >= kStages && !mbar_wait_bounded(&empty[s], ((i / kStages) - 1) & 1)) {
          raise_error(p.err, kErrTimeoutEmpty);
          *abort_flag = 1;
          break;
        }
        uint8_t* kt = stages + s * Smem::kStageBytes;
        uint8_t* vt = kt + Smem::kTileBytes;
        mbar_arrive_expect_tx(&full[s], Smem::kStageBytes);
        const int row = row0 + i * kTile;
        tma_load_2d(kt, &kmap, &full[s], 0, row);
        tma_load_2d(kt + kTile * 128, &kmap, &full[s], 64, row);
        tma_load_2d(vt, &vmap, &full[s], 0, row);
        tma_load_2d(vt + kTile * 128, &vmap, &full[s], 64, row);
      }
    }
  } else {
    // ======================= softmax / MMA warps (128 threads) =======================
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t q_addr = smem_u32(q_s), p_addr = smem_u32(p_s);
    const uint32_t idesc_s = idesc_bf16(false), idesc_o = idesc_bf16(true);
    float o[kMembers], l[kMembers];
#pragma unroll
    for (int c = 0; c < kMembers; ++c) o[c] = l[c] = 0.f;
    const float sl2 = p.scale_log2;
    int mma_phase = 0;
    for (int i = 0; i < tiles; ++i) {
      const int s = i % kStages;
      bool ok = mbar_wait_bounded(&full[s], (i / kStages) & 1);
      if (!ok) {
        raise_error(p.err, kErrTimeoutFull);
        *abort_flag = 1;
      }
      if (*abort_flag) break;
      uint8_t* kt = stages + s * Smem::kStageBytes;
      uint8_t* vt = kt + Smem::kTileBytes;
      const long long tile0 = begin + static_cast<long long>(i) * kTile;
      // ---- S^T = K_tile * Q^T : 8 UMMAs over D = 128 ----
      if (tid == 0) {
        tc_fence_after();
        const uint32_t k_addr = smem_u32(kt);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off_k = (kk >> 2) * (kTile * 128) + (kk & 3) * 32;
          const uint32_t off_q = (kk >> 2) * (kMembers * 128) + (kk & 3) * 32;
          umma_bf16(tmem_s, umma_desc(k_addr + off_k, 16, 1024), umma_desc(q_addr + off_q, 16, 1024), idesc_s,
                    kk > 0 ? 1u : 0u);
        }
        umma_commit(&mma_bar[0]);
      }
      if (!mbar_wait_bounded(&mma_bar[0], mma_phase)) {
        raise_error(p.err, kErrTimeoutMma);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      float sc[kMembers];
      tmem_ld32(tmem_s + lane_base, sc);
      // ---- mask, scale, column max ----
      const long long tok = tile0 + tid;
      const bool in_range = tok < stop;
#pragma unroll
      for (int c = 0; c < kMembers; ++c) {
        const bool visible = in_range && (tok < col_valid[c] || tok == col_own[c]);
        sc[c] = visible ? sc[c] * sl2 : -INFINITY;
      }
      const float wmax = transpose_reduce<true>(sc, lane);
      red[warp * kMembers + lane] = wmax;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (tid < kMembers) {
        float tmax = red[tid];
#pragma unroll
        for (int w = 1; w < kSoftmaxWarps; ++w) tmax = fmaxf(tmax, red[w * kMembers + tid]);
        const float old = col_max[tid];
        const float nm = fmaxf(old, tmax);
        const float piv = nm == -INFINITY ? 0.f : nm;
        col_piv[tid] = piv;
        col_corr[tid] = exp2f(old - piv);
        col_max[tid] = nm;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      // ---- P (bf16) into the K-major swizzled tile: row = member, column = token tid ----
      float corr[kMembers];
#pragma unroll
      for (int c = 0; c < kMembers; ++c) {
        const float pv = exp2f(sc[c] - col_piv[c]);
        corr[c] = col_corr[c];
        l[c] = l[c] * corr[c] + pv;
        const uint32_t off = (tid >> 6) * (kMembers * 128) + sw128(c, (tid & 63) >> 3) + (tid & 7) * 2;
        *reinterpret_cast<__nv_bfloat16*>(p_s + off) = __float2bfloat16_rn(pv);
      }
      if (!in_range) {
        // V row past the visible range: zero it so stale values never meet a zero weight.
        uint8_t* vrow0 = vt + tid * 128;
        uint8_t* vrow1 = vt + kTile * 128 + tid * 128;
#pragma unroll
        for (int c16 = 0; c16 < 8; ++c16) {
          *reinterpret_cast<uint4*>(vrow0 + c16 * 16) = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(vrow1 + c16 * 16) = make_uint4(0, 0, 0, 0);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      // ---- O^T_tile = V^T * P^T : 8 UMMAs over the 128 tokens ----
      if (tid == 0) {
        tc_fence_after();
        const uint32_t v_addr = smem_u32(vt);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off_v = kk * 16 * 128;  // 16 tokens = two 8-row groups
          const uint32_t off_p = (kk >> 2) * (kMembers * 128) + (kk & 3) * 32;
          umma_bf16(tmem_o, umma_desc(v_addr + off_v, kTile * 128, 1024), umma_desc(p_addr + off_p, 16, 1024),
                    idesc_o, kk > 0 ? 1u : 0u);
        }
        umma_commit(&mma_bar[1]);
      }
      if (!mbar_wait_bounded(&mma_bar[1], mma_phase)) {
        raise_error(p.err, kErrTimeoutMma);
        *abort_flag = 1;
        break;
      }
      mma_phase ^= 1;
      tc_fence_after();
      float ot[kMembers];
      tmem_ld32(tmem_o + lane_base, ot);
#pragma unroll
      for (int c = 0; c < kMembers; ++c) o[c] = o[c] * corr[c] + ot[c];
      // Both products of this stage are complete: hand the K/V buffers back to the producer.
      tc_fence_before();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (tid == 0) mbar_arrive(&empty[s]);
    }
    if (!*abort_flag) {
      // ---- denominators: per-member sums over the 128 token-threads ----
      const float wsum = transpose_reduce<false>(l, lane);
      red[warp * kMembers + lane] = wsum;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      // thread tid = dim d holds o[member] for this tile chunk; write partials or the output
      const int d = tid;
#pragma unroll
      for (int c = 0; c < kMembers; ++c) {
        const int m = group0 + c;
        if (m >= members) continue;
        const float L = red[c] + red[kMembers + c] + red[2 * kMembers + c] + red[3 * kMembers + c];
        const int t = m / G, g = m % G;
        if (p.splits == 1) {
          const size_t o_off = ((static_cast<size_t>(b) * T + t) * p.q_heads + h * G + g) * 128 + d;
          p.out[o_off] = __float2bfloat16_rn(L > 0.f ? o[c] / L : 0.f);
        } else {
          const size_t slot = (static_cast<size_t>(pair) * p.splits + split) * p.members_pad + m;
          p.acc[slot * 128 + d] = o[c];
          if (d == 0) p.stats[slot] = make_float2(col_max[c], L);
        }
      }
    }
  }
  // ---- teardown: every TMEM read and MMA has completed above; free the columns ----
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// LSE merge over KV splits, token-major output (decode_attention.py:455-478). One CTA per
// (row, token, query head); thread = dim.
__global__ void __launch_bounds__(128) verify_merge_kernel(const Params p) {
  pdl_wait();
  pdl_trigger();
  const int index = blockIdx.x;  // (b, t, hq) in output order
  const int hq = index % p.q_heads;
  const int t = (index / p.q_heads) % p.tokens;
  const int b = index / (p.q_heads * p.tokens);
  const int h = hq / p.groups, g = hq % p.groups;
  const int pair = b * p.kv_heads + h;
  const int m = t * p.groups + g;
  const int d = threadIdx.x;
  float M = -INFINITY;
  for (int s = 0; s < p.splits; ++s)
    M = fmaxf(M, p.stats[(static_cast<size_t>(pair) * p.splits + s) * p.members_pad + m].x);
  const float piv = M == -INFINITY ? 0.f : M;
  float L = 0.f, O = 0.f;
  for (int s = 0; s < p.splits; ++s) {
    const size_t slot = (static_cast<size_t>(pair) * p.splits + s) * p.members_pad + m;
    const float2 st = p.stats[slot];
    if (st.y == 0.f) continue;  // a split past the block saw nothing
    const float w = exp2f(st.x - piv);
    L += st.y * w;
    O += p.acc[slot * 128 + d] * w;
  }
  p.out[static_cast<size_t>(index) * 128 + d] = __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
}

}  // namespace verify
}  // namespace fb

using namespace fb;

extern "C" int fb_verify_attention_splits(int batch, int tokens, int kv_heads, int capacity) {
  if (batch <= 0 || kv_heads <= 0 || capacity <= 0) return 1;
  const int tiles = (capacity + verify::kTile - 1) / verify::kTile;
  const int want = (2 * sm_count() + batch * kv_heads - 1) / (batch * kv_heads);
  int s = want < 1 ? 1 : want;
  if (s > tiles) s = tiles;
  if (s > 64) s = 64;
  return s;
}

extern "C" size_t fb_verify_attention_workspace(int batch, int tokens, int q_heads, int kv_heads, int splits) {
  if (batch <= 0 || tokens <= 0 || q_heads <= 0 || kv_heads <= 0 || splits <= 0) return 0;
  const size_t members = static_cast<size_t>(tokens) * (q_heads / kv_heads);
  const size_t pad = (members + verify::kMembers - 1) / verify::kMembers * verify::kMembers;
  const size_t slots = static_cast<size_t>(batch) * kv_heads * splits * pad;
  return ((slots * 128 * sizeof(float) + 255) & ~size_t(255)) + slots * sizeof(float2);
}

extern "C" int fb_verify_attention(const void* q, const void* k, const void* v, const int64_t* position,
                                   const int64_t* chain, void* out, void* workspace, size_t workspace_bytes,
                                   int batch, int tokens, int q_heads, int kv_heads, int head_dim, int capacity,
                                   float scale, int splits, void* stream) {
  if (!q || !k || !v || !position || !chain || !out) return FB_ERR_ARG;
  if (batch <= 0 || tokens <= 0 || q_heads <= 0 || kv_heads <= 0 || capacity <= 0 || splits <= 0)
    return FB_ERR_ARG;
  if (head_dim != 128 || q_heads % kv_heads != 0) return FB_ERR_SHAPE;
  if (static_cast<long long>(batch) * kv_heads * capacity >= (1ll << 31)) return FB_ERR_SHAPE;
  if (batch * kv_heads > 65535 || splits > 65535) return FB_ERR_SHAPE;
  const int groups = q_heads / kv_heads;
  const int members = tokens * groups;
  const int member_groups = (members + verify::kMembers - 1) / verify::kMembers;
  if (member_groups > 64) return FB_ERR_SHAPE;
  if (splits > 1) {
    if (workspace == nullptr) return FB_ERR_ARG;
    if (workspace_bytes < fb_verify_attention_workspace(batch, tokens, q_heads, kv_heads, splits))
      return FB_ERR_WORKSPACE;
  }
  verify::Params p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.position = position;
  p.chain = chain;
  p.out = static_cast<__nv_bfloat16*>(out);
  const size_t pad = static_cast<size_t>(member_groups) * verify::kMembers;
  const size_t slots = static_cast<size_t>(batch) * kv_heads * splits * pad;
  p.acc = static_cast<float*>(workspace);
  p.stats = workspace ? reinterpret_cast<float2*>(static_cast<uint8_t*>(workspace) +
                                                  ((slots * 128 * sizeof(float) + 255) & ~size_t(255)))
                      : nullptr;
  p.batch = batch;
  p.tokens = tokens;
  p.q_heads = q_heads;
  p.kv_heads = kv_heads;
  p.groups = groups;
  p.capacity = capacity;
  p.splits = splits;
  const int per = (capacity + splits - 1) / splits;
  p.chunk = (per + verify::kTile - 1) / verify::kTile * verify::kTile;
  p.members_pad = static_cast<int>(pad);
  p.scale_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634);
  p.err = error_word();
  const uint64_t rows = static_cast<uint64_t>(batch) * kv_heads * capacity;
  CUtensorMap km, vm;
  int st = encode_bf16_2d(&km, k, rows, head_dim, head_dim, 64, verify::kTile, true);
  if (st != FB_OK) return st;
  st = encode_bf16_2d(&vm, v, rows, head_dim, head_dim, 64, verify::kTile, true);
  if (st != FB_OK) return st;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(verify::verify_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             verify::Smem::kTotal) != cudaSuccess)
      return FB_ERR_LAUNCH;
    configured[dev] = true;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  dim3 grid(batch * kv_heads, splits, member_groups);
  st = launch_ex(verify::verify_kernel, grid, dim3(verify::kThreads), verify::Smem::kTotal, s, 1, km, vm, p);
  if (st != FB_OK || splits == 1) return st;
  return launch_ex(verify::verify_merge_kernel, dim3(batch * tokens * q_heads), dim3(128), 0, s, 1, p);
}

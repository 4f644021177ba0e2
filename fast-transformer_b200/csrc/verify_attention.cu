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
//  * One CTA per (row, KV head, KV split, 32-member group), warp-specialized. A producer lane
//    streams 128-token K and V tiles with 2-D TMA (128-byte swizzle, no multicast) into a
//    3-stage ring; one lane of the MMA warp issues every UMMA and the warp owns TMEM.
//  * S^T = K_tile * Q^T is one tcgen05.mma chain (M = 128 tokens, N = 32 members, K = D)
//    with the fp32 accumulator in TMEM (double-buffered). Q sits in shared memory in the same
//    swizzled K-major layout, written once by the CTA.
//  * Eight softmax warps (TMEM lane quarter x half of the member columns; one token per
//    thread, 16 member columns) write P as bf16 into a K-major swizzled tile (double-buffered).
//  * Lazy pivot: a column's exponent pivot only moves when some score of a tile exceeds it by
//    more than 8 (log2 units, a factor of 256). One barrier-reduction vote per tile decides;
//    only then do the warps reduce the tile's column maxima (shuffle transpose-reduce and
//    shared memory) and rescale. P = 2^(s - pivot) then lies in (0, 256], which bf16 and fp32
//    hold exactly as well as (0, 1]; the result equals the reference's per-tile exact-maximum
//    form up to rounding.
//  * O^T_tile = V^T * P^T is a second tcgen05.mma chain (M = 128 dims, N = 32 members,
//    K = 128 tokens) with V read in place as an MN-major operand; each softmax thread (one dim)
//    folds the tile into its fp32 running output with the softmax correction, one tile behind
//    the scores, so the tensor core computes O(i-1) and S(i+1) while the warps work on tile i.
//  * head_dim 64 runs the same pipeline on the same 128-dim layout: TMA fills only the first
//    64-dim box of each K/V stage, the second box of every stage (and of Q) is zeroed once, so
//    the score product adds zeros and the value product's dims 64..127 come out zero and are
//    not stored.
//  * Every mbarrier wait is bounded; TMEM is freed on every path.
#include "tcgen05.cuh"

namespace fb {
namespace verify {

constexpr int kTile = 128;          // tokens per K/V tile (UMMA M of the score product)
constexpr int kMembers = 32;        // member columns per CTA (UMMA N)
constexpr int kStages = 3;          // K/V ring depth (64 KB stages)
constexpr int kSoftmaxWarps = 8;    // warp w: TMEM lanes 32*(w%4).., member columns 16*(w/4)..
constexpr int kHalf = kMembers / 2; // member columns per softmax warp
constexpr int kProducerWarp = kSoftmaxWarps;      // one lane issues every TMA
constexpr int kMmaWarp = kSoftmaxWarps + 1;       // one lane issues every UMMA; the warp owns TMEM
constexpr int kThreads = (kSoftmaxWarps + 2) * 32;
constexpr int kTmemCols = 4 * kMembers;  // S^T double buffer + O^T tile double buffer
constexpr float kSlack = 8.f;            // pivot moves when a score exceeds it by more (log2 units)

struct Params {
  const __nv_bfloat16* q;  // [B, T, Hq, D] token-major
  const int64_t* position; // [B]
  const int64_t* chain;    // [B]
  __nv_bfloat16* out;      // [B, T, Hq, D]
  float* acc;              // [pairs, S, members_pad, D] (splits > 1)
  float2* stats;           // [pairs, S, members_pad]
  int batch, tokens, q_heads, kv_heads, groups, capacity, splits, chunk, members_pad, dim;
  float scale_log2;
  unsigned* err;
};

// UMMA shapes: S^T = K * Q^T (M = 128 tokens, N = 32 members, A K-major) and
// O^T = V^T * P^T (M = 128 dims, N = 32 members, A = V read MN-major).
constexpr uint32_t kIdescS = tc::idesc_bf16(kTile, kMembers, false, false);
constexpr uint32_t kIdescO = tc::idesc_bf16(kTile, kMembers, true, false);
using tc::ex2_approx;

// True on every participating thread when `pred` is true on any of the `threads` threads that
// meet at named barrier `id` (bar.red.or: the barrier and the vote in one instruction).
__device__ __forceinline__ bool barrier_any(int id, int threads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred q, a;\n setp.ne.u32 q, %1, 0;\n bar.red.or.pred a, %2, %3, q;\n selp.u32 %0, 1, 0, a;\n}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(threads)
      : "memory");
  return r != 0;
}

// Column-wise reduction of a 32x16 block held one row per lane: afterwards lanes c and c+16
// hold the reduction of column c over all 32 rows (shuffle transpose-reduce, 16 shuffles).
template <bool kMax>
__device__ __forceinline__ float transpose_reduce16(const float (&v)[kHalf], int lane) {
  float a[kHalf];
#pragma unroll
  for (int i = 0; i < kHalf; ++i) a[i] = v[i];
#pragma unroll
  for (int width = kHalf / 2; width >= 1; width >>= 1) {
    const bool upper = (lane & width) != 0;
#pragma unroll
    for (int i = 0; i < width; ++i) {
      const float mine = upper ? a[width + i] : a[i];
      const float other = upper ? a[i] : a[width + i];
      const float recv = __shfl_xor_sync(0xffffffffu, other, width);
      a[i] = kMax ? fmaxf(mine, recv) : mine + recv;
    }
  }
  const float recv = __shfl_xor_sync(0xffffffffu, a[0], 16);
  return kMax ? fmaxf(a[0], recv) : a[0] + recv;
}

struct Smem {
  static constexpr int kTileBytes = 2 * kTile * 128;       // one of K or V: two 64-dim boxes
  static constexpr int kStageBytes = 2 * kTileBytes;       // K then V
  static constexpr int kQBytes = 2 * kMembers * 128;       // two 64-dim boxes of 32 rows
  static constexpr int kPBytes = 2 * kMembers * 128;       // one P tile: two 64-token boxes of 32 rows
  static constexpr int kRed = 2 * 4 * kMembers * 4;       // per-quarter column maxima, by tile parity
  static constexpr int kCol = 3 * kMembers * 4;            // run max, pivot, correction
  static constexpr int kMask = 2 * kMembers * 4;           // visibility limits per member
  static constexpr int kBars = (2 * kStages + 4 * 2) * 8;
  static constexpr int kTotal = 1024 + kStages * kStageBytes + kQBytes + 2 * kPBytes + kRed + kCol + kMask + kBars + 32;
  static_assert(kTotal <= 227 * 1024, "verify shared memory");
};

__global__ void __launch_bounds__(kThreads, 1)
    verify_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                  const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = base;
  uint8_t* q_s = base + kStages * Smem::kStageBytes;
  uint8_t* p_s = q_s + Smem::kQBytes;  // two P tiles
  float* red = reinterpret_cast<float*>(p_s + 2 * Smem::kPBytes);
  float* col_max = red + 2 * 4 * kMembers;   // running max per member (final, for split stats)
  float* col_piv = col_max + kMembers;
  float* col_corr = col_piv + kMembers;
  int* col_valid = reinterpret_cast<int*>(col_corr + kMembers);
  int* col_own = col_valid + kMembers;
  uint64_t* full = reinterpret_cast<uint64_t*>(col_own + kMembers);  // TMA -> MMA, per stage
  uint64_t* empty = full + kStages;                                   // MMA -> TMA, per stage
  uint64_t* s_full = empty + kStages;   // MMA -> softmax: S^T[b] holds a tile's scores
  uint64_t* s_free = s_full + 2;        // softmax -> MMA: S^T[b] has been read
  uint64_t* p_full = s_free + 2;        // softmax -> MMA: P[b] written
  uint64_t* o_full = p_full + 2;        // MMA -> softmax: O^T[b] holds a tile's product
  uint64_t* o_free = o_full + 2;        // softmax -> MMA: O^T[b] has been read
  uint64_t* done = o_free + 2;          // MMA lane: every issued UMMA has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int pair = blockIdx.x, split = blockIdx.y, group0 = blockIdx.z * kMembers;
  const int b = pair / p.kv_heads, h = pair % p.kv_heads;
  const int G = p.groups, T = p.tokens, members = T * G;

  // ---- set-up that reads nothing an earlier kernel writes: barriers, TMEM, zero boxes. It
  // overlaps the previous kernel's tail (programmatic dependent launch). ----
  if (warp == kProducerWarp && lane == 0) {
    for (int st = 0; st < kStages; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&s_free[x], kSoftmaxWarps);
      mbar_init(&p_full[x], kSoftmaxWarps);
      mbar_init(&o_full[x], 1);
      mbar_init(&o_free[x], kSoftmaxWarps);
    }
    mbar_init(done, 1);
    fence_barrier_init();
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    *abort_flag = 0;
    // The split's first ring-full of K/V rows into L2 while the previous kernel finishes
    // (which tiles are valid needs the position, read after the dependency wait).
    const int row0 = pair * p.capacity + split * p.chunk;
    for (int i = 0; i < kStages; ++i)
      for (int bx = 0; bx < p.dim / 64; ++bx) {
        tma_prefetch_l2_2d(&kmap, bx * 64, row0 + i * kTile);
        tma_prefetch_l2_2d(&vmap, bx * 64, row0 + i * kTile);
      }
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  const int D = p.dim;
  if (D == 64) {
    // head_dim 64: the second 64-dim box of every K and V stage stays zero (TMA never writes it)
    for (int e = tid; e < kStages * 2 * kTile * 8; e += blockDim.x) {
      const int st = e / (2 * kTile * 8), rest = e % (2 * kTile * 8);
      const int which = rest / (kTile * 8), c = rest % (kTile * 8);
      *reinterpret_cast<uint4*>(stages + st * Smem::kStageBytes + which * Smem::kTileBytes + kTile * 128 + c * 16) =
          make_uint4(0, 0, 0, 0);
    }
  }
  // ---- after the dependency wait: positions, chains and Q come from earlier kernels ----
  pdl_wait();
  pdl_trigger();
  // Every global read of the set-up is issued before the first shared-memory store (one round
  // trip): the row's position and chain, and this thread's Q chunks.
  const long long position_b = p.position[b];
  const long long chain_b = p.chain[b];
  constexpr int kQChunks = kMembers * 16;  // 16-byte chunks of the 32-member Q tile
  constexpr int kQPerThread = (kQChunks + kThreads - 1) / kThreads;
  uint4 qv[kQPerThread];
#pragma unroll
  for (int it = 0; it < kQPerThread; ++it) {
    const int e = tid + it * kThreads;
    const int r = e / 16, c16 = e % 16;  // member row, 16-byte chunk of the 128-dim layout
    const int m = group0 + r;
    qv[it] = make_uint4(0, 0, 0, 0);
    if (e < kQChunks && m < members && c16 * 8 < D) {
      const int t = m / G, g = m % G;
      qv[it] = *reinterpret_cast<const uint4*>(p.q + ((static_cast<size_t>(b) * T + t) * p.q_heads + h * G + g) * D +
                                               c16 * 8);
    }
  }
  const long long first = position_b + 1;                 // first block token's slot + 1
  long long end = first + T - 1;                          // one past the last block slot
  if (end > p.capacity) end = p.capacity;
  const long long begin = static_cast<long long>(split) * p.chunk;
  long long stop = begin + p.chunk;
  if (stop > end) stop = end;
  const int tiles = stop > begin ? static_cast<int>((stop - begin + kTile - 1) / kTile) : 0;
  // Q members [group0, group0 + 32) of this (row, KV head) into the swizzled K-major tile;
  // rows past the real members, and dims past D, are zero.
#pragma unroll
  for (int it = 0; it < kQPerThread; ++it) {
    const int e = tid + it * kThreads;
    if (e < kQChunks) {
      const int r = e / 16, c16 = e % 16;
      *reinterpret_cast<uint4*>(q_s + (c16 >> 3) * (kMembers * 128) + sw128(r, c16 & 7)) = qv[it];
    }
  }
  if (tid < kMembers) {
    const int m = group0 + tid;
    const int t = m / G;
    const bool live = m < members;
    const bool chained = live && t < chain_b;
    col_valid[tid] = live ? static_cast<int>(first + (chained ? t : 0)) : 0;
    col_own[tid] = live && !chained ? static_cast<int>(first - 1 + t) : -1;
    col_max[tid] = -INFINITY;
  }
  fence_proxy_async_smem();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  // S^T[x] = columns [32x, 32x + 32); O^T[x] = columns [64 + 32x, 96 + 32x)

  if (warp == kProducerWarp) {
    // ============================ TMA producer ============================
    if (lane == 0) {
      const int row0 = pair * p.capacity + static_cast<int>(begin);
      for (int i = 0; i < tiles && !*abort_flag; ++i) {
        const int st = i % kStages;
        if (i >= kStages && !mbar_wait_bounded(&empty[st], ((i / kStages) - 1) & 1)) {
          raise_error(p.err, kErrTimeoutEmpty);
          *abort_flag = 1;
          break;
        }
        uint8_t* kt = stages + st * Smem::kStageBytes;
        uint8_t* vt = kt + Smem::kTileBytes;
        mbar_arrive_expect_tx(&full[st], D == 128 ? Smem::kStageBytes : Smem::kStageBytes / 2);
        const int row = row0 + i * kTile;
        tma_load_2d(kt, &kmap, &full[st], 0, row);
        tma_load_2d(vt, &vmap, &full[st], 0, row);
        if (D == 128) {
          tma_load_2d(kt + kTile * 128, &kmap, &full[st], 64, row);
          tma_load_2d(vt + kTile * 128, &vmap, &full[st], 64, row);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ============================ UMMA issuer ============================
    if (lane == 0) {
      const uint32_t q_addr = smem_u32(q_s), p_addr = smem_u32(p_s);
      const uint32_t idesc_s = kIdescS, idesc_o = kIdescO;
      auto issue_o = [&](int j) {
        const int x = j & 1;
        tc::fence_after();
        const uint32_t v_addr = smem_u32(stages + (j % kStages) * Smem::kStageBytes + Smem::kTileBytes);
        const uint32_t pb = p_addr + x * Smem::kPBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off_v = kk * 16 * 128;  // 16 tokens = two 8-row groups
          const uint32_t off_p = (kk >> 2) * (kMembers * 128) + (kk & 3) * 32;
          tc::mma_bf16(tmem + 64 + 32 * x, tc::desc_sw128(v_addr + off_v, kTile * 128, 1024), tc::desc_sw128(pb + off_p, 16, 1024),
                    idesc_o, kk > 0 ? 1u : 0u);
        }
        tc::commit(&o_full[x]);
        tc::commit(&empty[j % kStages]);  // both products of tile j read their K/V stage
      };
      // S(i) needs tile i's K/V stage and S^T[i % 2] read by the softmax (tile i - 2); O(j)
      // needs P(j) and O^T[j % 2] folded (tile j - 2). The lane issues whichever is ready first,
      // so a tile's value product (and with it the release of its K/V stage to the TMA lane)
      // never waits for the next tile's data. S runs at most two tiles ahead of O.
      auto issue_s = [&](int i) {
        const int st = i % kStages, x = i & 1;
        tc::fence_after();
        const uint32_t k_addr = smem_u32(stages + st * Smem::kStageBytes);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off_k = (kk >> 2) * (kTile * 128) + (kk & 3) * 32;
          const uint32_t off_q = (kk >> 2) * (kMembers * 128) + (kk & 3) * 32;
          tc::mma_bf16(tmem + 32 * x, tc::desc_sw128(k_addr + off_k, 16, 1024), tc::desc_sw128(q_addr + off_q, 16, 1024), idesc_s,
                    kk > 0 ? 1u : 0u);
        }
        tc::commit(&s_full[x]);
      };
      bool ok = true;
      int next_s = 0, next_o = 0;
      unsigned long long idle_since = 0;
      while (ok && next_o < tiles && !*abort_flag) {
        bool progressed = false;
        if (next_s < tiles && next_s <= next_o + 2) {
          const int i = next_s, x = i & 1;
          if (mbar_test(&full[i % kStages], (i / kStages) & 1) &&
              (i < 2 || mbar_test(&s_free[x], ((i - 2) >> 1) & 1))) {
            issue_s(i);
            ++next_s;
            progressed = true;
          }
        }
        if (next_o < next_s) {
          const int j = next_o, x = j & 1;
          if (mbar_test(&p_full[x], (j >> 1) & 1) && (j < 2 || mbar_test(&o_free[x], ((j - 2) >> 1) & 1))) {
            issue_o(j);
            ++next_o;
            progressed = true;
          }
        }
        if (progressed) {
          idle_since = 0;
        } else if (idle_since == 0) {
          idle_since = globaltimer();
        } else if (globaltimer() - idle_since > kWaitBudgetNs) {
          ok = false;
        }
      }
      if (!ok) {
        raise_error(p.err, kErrTimeoutMma);
        *abort_flag = 1;
      }
      // every UMMA issued above has completed before TMEM can be freed
      tc::commit(done);
      if (!mbar_wait_bounded(done, 0)) raise_error(p.err, kErrTimeoutDrain);
    }
    __syncwarp();
  } else {
    // ======================= softmax warps (256 threads) =======================
    // Warp w reads TMEM lanes 32*(w%4).. (tokens of S^T, dims of O^T) and member columns
    // [16*(w/4), 16*(w/4) + 16): two warps per scheduler, 16 columns per thread.
    const int quarter = warp & 3, half = warp >> 2;
    const int row = quarter * 32 + lane;  // token of the S^T tile, dim of the O^T tile
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int col0 = half * kHalf;
    float o[kHalf], l[kHalf], corr_prev[kHalf], run_max[kHalf];
#pragma unroll
    for (int c = 0; c < kHalf; ++c) {
      o[c] = l[c] = corr_prev[c] = 0.f;
      run_max[c] = -INFINITY;
    }
    const float sl2 = p.scale_log2;
    // o <- o * corr(j) + O^T(j): the product of tile j, read from TMEM once it is complete
    auto fold = [&](int j) -> bool {
      const int x = j & 1;
      if (!mbar_wait_bounded(&o_full[x], (j >> 1) & 1)) return false;
      tc::fence_after();
      float ot[kHalf];
      tc::ld16(tmem + 64 + 32 * x + col0 + lane_base, ot);
      tc::fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[x]);
#pragma unroll
      for (int c = 0; c < kHalf; ++c) o[c] = o[c] * corr_prev[c] + ot[c];
      return true;
    };
    bool ok = true;
    for (int i = 0; i < tiles; ++i) {
      const int x = i & 1;
      if (*abort_flag || !mbar_wait_bounded(&s_full[x], (i >> 1) & 1)) {
        ok = false;
        break;
      }
      tc::fence_after();
      float sc[kHalf];
      tc::ld16(tmem + 32 * x + col0 + lane_base, sc);
      tc::fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[x]);
      const long long tile0 = begin + static_cast<long long>(i) * kTile;
      uint8_t* vt = stages + (i % kStages) * Smem::kStageBytes + Smem::kTileBytes;
      // ---- mask, scale, column max. A tile wholly below the block's first slot is visible
      // to every live member (dead members' columns only ever reach their own, unused,
      // outputs), so only the block's own tile pays the per-member masks. ----
      const long long tok = tile0 + row;
      const bool in_range = tok < stop;
      if (tile0 + kTile <= first - 1 && tile0 + kTile <= stop) {
#pragma unroll
        for (int c = 0; c < kHalf; ++c) sc[c] *= sl2;
      } else {
#pragma unroll
        for (int c = 0; c < kHalf; ++c) {
          const bool visible = in_range && (tok < col_valid[col0 + c] || tok == col_own[col0 + c]);
          sc[c] = visible ? sc[c] * sl2 : -INFINITY;
        }
      }
      // Lazy pivot: every thread votes whether one of its scores exceeds the column's pivot
      // by more than kSlack (a column that has seen only -inf has pivot -inf, so any finite
      // score votes). Only a tile that some thread votes for reduces its column maxima: each
      // quarter's max over its 32 tokens goes to red[parity][quarter], and after one barrier
      // every thread folds the four quarters and its running max itself (all threads of a
      // column half compute the same values). red is double-buffered by tile parity.
      bool need = false;
#pragma unroll
      for (int c = 0; c < kHalf; ++c) need |= sc[c] > run_max[c] + kSlack;
      float piv[kHalf], corr[kHalf];
      if (barrier_any(1, 256, need)) {
        const float wmax = transpose_reduce16<true>(sc, lane);
        float* rq = red + x * 4 * kMembers;
        if (lane < kHalf) rq[quarter * kMembers + col0 + lane] = wmax;
        asm volatile("bar.sync 1, 256;" ::: "memory");
#pragma unroll
        for (int c4 = 0; c4 < kHalf / 4; ++c4) {
          float4 t4 = *reinterpret_cast<const float4*>(rq + col0 + 4 * c4);
#pragma unroll
          for (int w = 1; w < 4; ++w) {
            const float4 u4 = *reinterpret_cast<const float4*>(rq + w * kMembers + col0 + 4 * c4);
            t4.x = fmaxf(t4.x, u4.x), t4.y = fmaxf(t4.y, u4.y), t4.z = fmaxf(t4.z, u4.z), t4.w = fmaxf(t4.w, u4.w);
          }
          const float tm[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int c = 4 * c4 + e;
            const float nm = fmaxf(run_max[c], tm[e]);
            piv[c] = nm == -INFINITY ? 0.f : nm;
            // an unchanged max rescales by exactly 1 (and an all -inf column has l = o = 0)
            corr[c] = nm == run_max[c] ? 1.f : ex2_approx(run_max[c] - piv[c]);
            run_max[c] = nm;
          }
        }
      } else {
#pragma unroll
        for (int c = 0; c < kHalf; ++c) {
          piv[c] = run_max[c] == -INFINITY ? 0.f : run_max[c];
          corr[c] = 1.f;
        }
      }
      // ---- P (bf16) into P[x], K-major swizzled: row = member, column = token. P[x] was
      // last read by O(i-2), whose completion fold(i-2) already waited for. ----
      uint8_t* pt = p_s + x * Smem::kPBytes;
      const uint32_t pcol = (row >> 6) * (kMembers * 128) + (row & 7) * 2;
#pragma unroll
      for (int c = 0; c < kHalf; ++c) {
        const float pv = ex2_approx(sc[c] - piv[c]);
        l[c] = l[c] * corr[c] + pv;
        *reinterpret_cast<__nv_bfloat16*>(pt + pcol + sw128(col0 + c, (row & 63) >> 3)) = __float2bfloat16_rn(pv);
      }
      if (!in_range && half == 0) {
        // V row past the visible range: zero it so stale values never meet a zero weight.
        uint8_t* vrow0 = vt + row * 128;
        uint8_t* vrow1 = vt + kTile * 128 + row * 128;
#pragma unroll
        for (int c16 = 0; c16 < 8; ++c16) {
          *reinterpret_cast<uint4*>(vrow0 + c16 * 16) = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(vrow1 + c16 * 16) = make_uint4(0, 0, 0, 0);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[x]);
      // fold the previous tile's product (computed while this tile's softmax ran)
      if (i >= 1 && !fold(i - 1)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int c = 0; c < kHalf; ++c) corr_prev[c] = corr[c];
    }
    if (ok && tiles >= 1 && !*abort_flag) ok = fold(tiles - 1);
    if (!ok) {
      raise_error(p.err, kErrTimeoutMma);
      *abort_flag = 1;
    }
    if (!*abort_flag) {
      // ---- denominators: per-member sums over the 128 token rows; the final maxima ----
      if (quarter == 0) {
#pragma unroll
        for (int c = 0; c < kHalf; ++c)
          if (lane == c) col_max[col0 + c] = run_max[c];
      }
      const float wsum = transpose_reduce16<false>(l, lane);
      asm volatile("bar.sync 1, 256;" ::: "memory");  // every thread is past its last max read
      if (lane < kHalf) red[quarter * kMembers + col0 + lane] = wsum;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      // thread (dim d = row, members col0..col0+15) writes partials or the output
      const int d = row;
#pragma unroll
      for (int c = 0; c < kHalf; ++c) {
        const int m = group0 + col0 + c;
        if (m >= members || d >= D) continue;
        const int mc = col0 + c;
        const float L = red[mc] + red[kMembers + mc] + red[2 * kMembers + mc] + red[3 * kMembers + mc];
        const int t = m / G, g = m % G;
        if (p.splits == 1) {
          const size_t o_off = ((static_cast<size_t>(b) * T + t) * p.q_heads + h * G + g) * D + d;
          p.out[o_off] = __float2bfloat16_rn(L > 0.f ? o[c] / L : 0.f);
        } else {
          const size_t slot = (static_cast<size_t>(pair) * p.splits + split) * p.members_pad + m;
          p.acc[slot * 128 + d] = o[c];
          if (d == 0) p.stats[slot] = make_float2(col_max[mc], L);
        }
      }
    }
  }
  // ---- teardown: the MMA lane saw every UMMA complete and every TMEM read has waited ----
  tc::fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc::fence_after();
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
  if (d >= p.dim) return;
  // up to kMergeSplits splits: every load in flight at once (one L2 round trip)
  constexpr int kMergeSplits = 4;
  float L = 0.f, O = 0.f;
  const size_t slot0 = static_cast<size_t>(pair) * p.splits * p.members_pad + m;  // split s: + s * members_pad
  if (p.splits <= kMergeSplits) {
    float2 st[kMergeSplits];
    float a[kMergeSplits];
#pragma unroll
    for (int s = 0; s < kMergeSplits; ++s) {
      const size_t slot = slot0 + static_cast<size_t>(s) * p.members_pad;
      st[s] = s < p.splits ? p.stats[slot] : make_float2(-INFINITY, 0.f);
      a[s] = s < p.splits ? p.acc[slot * 128 + d] : 0.f;
    }
    float M = -INFINITY;
#pragma unroll
    for (int s = 0; s < kMergeSplits; ++s) M = fmaxf(M, st[s].x);
    const float piv = M == -INFINITY ? 0.f : M;
#pragma unroll
    for (int s = 0; s < kMergeSplits; ++s) {
      if (st[s].y == 0.f) continue;  // a split past the block (or past p.splits) saw nothing
      const float w = exp2f(st[s].x - piv);
      L += st[s].y * w;
      O += a[s] * w;
    }
  } else {
    float M = -INFINITY;
    for (int s = 0; s < p.splits; ++s) M = fmaxf(M, p.stats[slot0 + static_cast<size_t>(s) * p.members_pad].x);
    const float piv = M == -INFINITY ? 0.f : M;
    for (int s = 0; s < p.splits; ++s) {
      const size_t slot = slot0 + static_cast<size_t>(s) * p.members_pad;
      const float2 st = p.stats[slot];
      if (st.y == 0.f) continue;  // a split past the block saw nothing
      const float w = exp2f(st.x - piv);
      L += st.y * w;
      O += p.acc[slot * 128 + d] * w;
    }
  }
  p.out[static_cast<size_t>(index) * p.dim + d] = __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
}

}  // namespace verify
}  // namespace fb

using namespace fb;

extern "C" int fb_verify_attention_splits(int batch, int tokens, int kv_heads, int capacity) {
  if (batch <= 0 || kv_heads <= 0 || capacity <= 0) return 1;
  // One CTA per SM (the 3-stage ring fills shared memory). Model the time as waves x (tiles
  // per CTA + ~2 tiles of fixed cost: TMEM allocation, Q staging, the first TMA round trip)
  // and take the cheapest split count (config 5, 64 pairs x 33 tiles: 2 splits, one wave).
  const int tiles = (capacity + verify::kTile - 1) / verify::kTile;
  const long long pairs = static_cast<long long>(batch) * kv_heads;
  const int sms = sm_count();
  int best = 1;
  long long best_cost = -1;
  for (int s = 1; s <= tiles && s <= 64; ++s) {
    const long long waves = (pairs * s + sms - 1) / sms;
    const long long cost = waves * ((tiles + s - 1) / s + 2);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
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
  if ((head_dim != 64 && head_dim != 128) || q_heads % kv_heads != 0) return FB_ERR_SHAPE;
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
  p.dim = head_dim;
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

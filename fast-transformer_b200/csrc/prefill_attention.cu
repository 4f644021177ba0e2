// Causal GQA prefill attention (flash attention forward) on the 5th-generation tensor cores
// (sm_100a).
//
// Replaces the reference's prefill path, engine/attention.py:8-21 (`grouped_sdpa` with no
// mask: torch SDPA's Flash backend, is_causal, enable_gqa): for every query token t of a row
// and query head hq, softmax(q . k_j * scale) over keys j <= t of KV head hq / G, times V,
// with fp32 scores and accumulation and P rounded to bf16 for the value product.
//
// B200 design (one CTA per (pair of 128-query tiles, query head, row); heaviest pairs first):
//  * The two query tiles A and B (256 consecutive queries) share every K/V tile. A TMA lane
//    loads both Q tiles once and streams 128-key K tiles and V tiles through separate 2-stage
//    rings (128-byte swizzle, no multicast).
//  * A UMMA lane issues S_X = Q_X K^T (M = N = 128, K = D) into tile X's TMEM columns and
//    O_X += P_X V (M = 128, N = D, K = 128 keys) with P_X read from TMEM - the softmax wrote it
//    as bf16 pairs over S_X's first 64 columns - and V read MN-major from shared memory. Per key
//    tile j the order is O_A(j), S_A(j+1), O_B(j), S_B(j+1): one tile's softmax overlaps the
//    other tile's products, and each commit also covers every product issued before it.
//  * Two softmax warpgroups (tile A: warps 0-3, tile B: warps 4-7), one thread per query row
//    holding its 128 scores in registers: row max, lazy rescale (the pivot moves only when the
//    max grows by more than 8 in log2 units; O is then rescaled in TMEM), P = 2^(s - pivot)
//    rounded to bf16, row sum. Tiles below the diagonal skip the masks.
//  * Every mbarrier wait is bounded; TMEM is freed on every path.
#include "tcgen05.cuh"

namespace fb {
namespace prefill {

constexpr int kTile = 128;          // queries per tile and keys per K/V tile
constexpr int kSoftmaxWarps = 8;    // warps 0-3: tile A rows, 4-7: tile B rows
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 10 * 32;
constexpr int kTmemCols = 512;      // S_A, S_B (128 each), O_A, O_B (D each)
constexpr float kRescaleAbove = 8.0f;  // log2 units

struct Params {
  __nv_bfloat16* out;  // [B, T, Hq, D]
  int batch, tokens, q_heads, kv_heads, groups, capacity;
  float scale_log2;
  unsigned* err;
};

template <int D>
struct Smem {
  static constexpr int kBox = kTile * 128;            // 128 rows x 64 bf16 (one 128-byte row each)
  static constexpr int kTileBytes = (D / 64) * kBox;  // 128 rows x D (Q, K or V)
  static constexpr int kQOff = 0;                     // Q_A, Q_B
  static constexpr int kKOff = 2 * kTileBytes;        // K ring, 2 stages
  static constexpr int kVOff = kKOff + 2 * kTileBytes;  // V ring, 2 stages
  static constexpr int kBarOff = kVOff + 2 * kTileBytes;
  static constexpr int kBars = 16;
  static constexpr int kTotal = 1024 + kBarOff + kBars * 8 + 16;
  static_assert(kTotal <= 227 * 1024, "prefill shared memory");
};

// Packs two fp32 values as bf16 (lo, hi) into one 32-bit TMEM column.
__device__ __forceinline__ uint32_t pack2(float lo, float hi) { return pack_bf16x2(lo, hi); }

// Writes 32 consecutive 32-bit columns of this warp's 32 TMEM lanes (no wait).
__device__ __forceinline__ void st32u(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// 32 consecutive 32-bit columns of this warp's 32 TMEM lanes, without waiting for the load.
__device__ __forceinline__ void ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// UMMA with A = P in tensor memory (M = 128 rows, K = 16 per step) and B from shared memory.
__device__ __forceinline__ void mma_bf16_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

template <int D>
// 200 registers per thread: the softmax rows hold 128 scores; 320 x 200 fits one CTA per SM.
__global__ void __maxnreg__(200)
    prefill_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, const Params p) {
  using S = Smem<D>;
  constexpr uint32_t kIdescS = tc::idesc_bf16(kTile, kTile, false, false);
  constexpr uint32_t kIdescO = tc::idesc_bf16(kTile, D, false, true);
  pdl_wait();
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = base + S::kQOff;
  uint8_t* k_s = base + S::kKOff;
  uint8_t* v_s = base + S::kVOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + S::kBarOff);
  uint64_t* k_full = bars;       // [2] K stage landed
  uint64_t* k_empty = bars + 2;  // [2] K stage read by its score products
  uint64_t* v_full = bars + 4;   // [2] V stage landed
  uint64_t* v_empty = bars + 6;  // [2] V stage read by its value products
  uint64_t* s_full = bars + 8;   // [tile] S_X computed (and every earlier product complete)
  uint64_t* p_full = bars + 10;  // [tile] P_X written over S_X (four warps)
  uint64_t* q_full = bars + 12;
  uint64_t* done = bars + 13;    // every product issued has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q_tiles = (p.tokens + kTile - 1) / kTile;
  const int pairs = (q_tiles + 1) / 2;
  const int qp = pairs - 1 - static_cast<int>(blockIdx.x);  // the heaviest (latest) pairs first
  const int qa = 2 * qp;                                    // tile A; tile B = qa + 1
  const bool has_b = (qa + 1) * kTile < p.tokens;
  const int hq = blockIdx.y, b = blockIdx.z;
  const int hkv = hq / p.groups;
  const int last_j = has_b ? qa + 1 : qa;  // key tiles [0, last_j]; tile A stops at qa

  if (warp == kProducerWarp && lane == 0) {
    for (int x = 0; x < 2; ++x) {
      mbar_init(&k_full[x], 1);
      mbar_init(&k_empty[x], 1);
      mbar_init(&v_full[x], 1);
      mbar_init(&v_empty[x], 1);
      mbar_init(&s_full[x], 1);
      mbar_init(&p_full[x], 4);  // the tile's four softmax warps
    }
    mbar_init(q_full, 1);
    mbar_init(done, 1);
    fence_barrier_init();
    prefetch_tensormap(&qmap);
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    *abort_flag = 0;
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  // tile X: S_X at columns [128 X, 128 X + 128), O_X at [256 + D X, 256 + D X + D)

  if (warp == kProducerWarp) {
    // ============================ TMA producer ============================
    if (lane == 0) {
      const int qrow = (b * p.q_heads + hq) * p.tokens + qa * kTile;
      mbar_arrive_expect_tx(q_full, (has_b ? 2 : 1) * S::kTileBytes);
#pragma unroll
      for (int bx = 0; bx < D / 64; ++bx) {
        tma_load_2d(q_s + bx * S::kBox, &qmap, q_full, bx * 64, qrow);
        if (has_b) tma_load_2d(q_s + S::kTileBytes + bx * S::kBox, &qmap, q_full, bx * 64, qrow + kTile);
      }
      const int kvrow = (b * p.kv_heads + hkv) * p.capacity;
      for (int j = 0; j <= last_j && !*abort_flag; ++j) {
        const int st = j & 1;
        const int row = kvrow + j * kTile;
        if (j >= 2 && !mbar_wait_bounded(&k_empty[st], ((j - 2) >> 1) & 1)) {
          raise_error(p.err, kErrTimeoutEmpty);
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&k_full[st], S::kTileBytes);
#pragma unroll
        for (int bx = 0; bx < D / 64; ++bx)
          tma_load_2d(k_s + st * S::kTileBytes + bx * S::kBox, &kmap, &k_full[st], bx * 64, row);
        if (j >= 2 && !mbar_wait_bounded(&v_empty[st], ((j - 2) >> 1) & 1)) {
          raise_error(p.err, kErrTimeoutEmpty);
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&v_full[st], S::kTileBytes);
#pragma unroll
        for (int bx = 0; bx < D / 64; ++bx)
          tma_load_2d(v_s + st * S::kTileBytes + bx * S::kBox, &vmap, &v_full[st], bx * 64, row);
      }
    }
  } else if (warp == kMmaWarp) {
    // ============================ UMMA issuer ============================
    // Every lane takes the waits (the warp zeroes V rows past the prompt); lane 0 issues.
    const uint32_t q_addr = smem_u32(q_s);
    auto issue_s = [&](int x, int j) {
      const uint32_t k_addr = smem_u32(k_s + (j & 1) * S::kTileBytes);
      const uint32_t qx = q_addr + x * S::kTileBytes;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = (kk >> 2) * S::kBox + (kk & 3) * 32;  // 16 dims of the 128-byte rows
        tc::mma_bf16(tmem + 128 * x, tc::desc_sw128(qx + off, 16, 1024), tc::desc_sw128(k_addr + off, 16, 1024),
                     kIdescS, kk > 0 ? 1u : 0u);
      }
      tc::commit(&s_full[x]);
    };
    auto issue_o = [&](int x, int j) {
      const uint32_t v_addr = smem_u32(v_s + (j & 1) * S::kTileBytes);
#pragma unroll
      for (int kk = 0; kk < kTile / 16; ++kk) {
        // P: 16 keys = 8 packed columns of S_X; V: 16 key rows, MN-major over D
        mma_bf16_tmem_a(tmem + 256 + D * x, tmem + 128 * x + 8 * kk,
                        tc::desc_sw128(v_addr + kk * 16 * 128, S::kBox, 1024), kIdescO, (j > 0 || kk > 0) ? 1u : 0u);
      }
    };
    bool ok = mbar_wait_bounded(q_full, 0) && mbar_wait_bounded(&k_full[0], 0);
    if (ok && lane == 0) {
      tc::fence_after();
      issue_s(0, 0);
      if (has_b) issue_s(1, 0);
      tc::commit(&k_empty[0]);
    }
    for (int j = 0; j <= last_j && ok; ++j) {
      const int st = j & 1;
      ok = mbar_wait_bounded(&v_full[st], (j >> 1) & 1);
      if (!ok || *abort_flag) break;
      if (j * kTile + kTile > p.tokens) {
        // keys past the prompt: zero their V rows, so stale cache values never meet P = 0
        uint8_t* vt = v_s + st * S::kTileBytes;
        const int first = p.tokens - j * kTile;
        for (int e = lane; e < (kTile - first) * (D / 8); e += 32) {
          const int r = first + e / (D / 8), c16 = e % (D / 8);
          *reinterpret_cast<uint4*>(vt + (c16 >> 3) * S::kBox + r * 128 + (c16 & 7) * 16) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
        __syncwarp();
      }
      const bool a_live = j <= qa;
      const bool next_a = j + 1 <= qa, next_b = has_b && j + 1 <= last_j;
      if (a_live) ok = mbar_wait_bounded(&p_full[0], j & 1);
      if (ok && (next_a || next_b)) ok = mbar_wait_bounded(&k_full[(j + 1) & 1], ((j + 1) >> 1) & 1);
      if (!ok) break;
      if (lane == 0) {
        tc::fence_after();
        if (a_live) issue_o(0, j);
        if (next_a) issue_s(0, j + 1);
      }
      if (has_b) {
        ok = mbar_wait_bounded(&p_full[1], j & 1);
        if (!ok) break;
        if (lane == 0) {
          tc::fence_after();
          issue_o(1, j);
          if (next_b) issue_s(1, j + 1);
        }
      }
      if (lane == 0) {
        if (next_a || next_b) tc::commit(&k_empty[(j + 1) & 1]);
        tc::commit(&v_empty[st]);
      }
      __syncwarp();
    }
    if (!ok) {
      if (lane == 0) raise_error(p.err, kErrTimeoutMma);
      *abort_flag = 1;
    }
    if (lane == 0) {
      tc::commit(done);  // arrives once every product issued above has completed
      if (!mbar_wait_bounded(done, 0)) raise_error(p.err, kErrTimeoutDrain);
    }
    __syncwarp();
  } else {
    // ============================ softmax warps ============================
    // Warp w handles tile X = w / 4, TMEM lanes 32*(w%4).. = its query rows; one thread per row.
    // Control flow stays warp-uniform: tcgen05.ld/st are .sync.aligned.
    const int x = warp >> 2, quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int t = (qa + x) * kTile + row;  // this row's token
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_addr = tmem + 128 * x + lane_base;
    const uint32_t o_addr = tmem + 256 + D * x + lane_base;
    const float sl2 = p.scale_log2;
    const int last_key = min(t, p.tokens - 1);  // keys <= last_key are visible to this row
    const int my_last = qa + x;                 // this tile's diagonal key tile
    const bool live_tile = x == 0 || has_b;
    float pivot = -INFINITY, lsum = 0.f;
    bool ok = true;
    for (int j = 0; live_tile && j <= my_last; ++j) {
      const bool waited = !*abort_flag && mbar_wait_bounded(&s_full[x], j & 1);
      if (!__all_sync(0xffffffffu, waited)) {
        ok = false;
        break;
      }
      tc::fence_after();
      float v[128];
      {
        uint32_t r0[32], r1[32], r2[32], r3[32];
        ld32_nowait(s_addr, r0);
        ld32_nowait(s_addr + 32, r1);
        ld32_nowait(s_addr + 64, r2);
        ld32_nowait(s_addr + 96, r3);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          v[c] = __uint_as_float(r0[c]);
          v[32 + c] = __uint_as_float(r1[c]);
          v[64 + c] = __uint_as_float(r2[c]);
          v[96 + c] = __uint_as_float(r3[c]);
        }
      }
      // a tile wholly below the diagonal and inside the prompt is visible to every row
      const bool interior = j < qa + x && j * kTile + kTile <= p.tokens;
      const int key0 = j * kTile;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        v[c] = (interior || key0 + c <= last_key) ? v[c] * sl2 : -INFINITY;
        mx = fmaxf(mx, v[c]);
      }
      float corr = 1.f;
      const bool need = mx > pivot + kRescaleAbove || (pivot == -INFINITY && mx > -INFINITY);
      if (need) {
        corr = pivot == -INFINITY ? 0.f : tc::ex2_approx(pivot - mx);
        pivot = mx;
      }
      lsum *= corr;
      if (j >= 1 && __any_sync(0xffffffffu, need)) {
        // O_X holds the products through tile j - 1, complete: s_full(j) covers them
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          float o[32];
          tc::ld32(o_addr + c0, o);
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] *= corr;
          tc::st32(o_addr + c0, o);
        }
      }
      const float piv = pivot == -INFINITY ? 0.f : pivot;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t packed[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float p0 = tc::ex2_approx(v[64 * h + 2 * c] - piv);   // -inf gives 0
          const float p1 = tc::ex2_approx(v[64 * h + 2 * c + 1] - piv);
          lsum += p0 + p1;
          packed[c] = pack2(p0, p1);
        }
        st32u(s_addr + 32 * h, packed);  // P keys [64 h, 64 h + 64) as 32 packed columns
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc::fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[x]);
    }
    // every product has completed before the output is read
    if (ok && live_tile) ok = __all_sync(0xffffffffu, mbar_wait_bounded(done, 0));
    if (!ok) {
      raise_error(p.err, kErrTimeoutMma);
      *abort_flag = 1;
    }
    if (ok && live_tile) {
      tc::fence_after();
      const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
      __nv_bfloat16* dst = p.out + ((static_cast<size_t>(b) * p.tokens + t) * p.q_heads + hq) * D;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 32) {
        float o[32];
        tc::ld32(o_addr + c0, o);
        if (t < p.tokens) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(dst + c0 + 8 * q) = make_uint4(
                pack_bf16x2(o[8 * q] * inv, o[8 * q + 1] * inv), pack_bf16x2(o[8 * q + 2] * inv, o[8 * q + 3] * inv),
                pack_bf16x2(o[8 * q + 4] * inv, o[8 * q + 5] * inv), pack_bf16x2(o[8 * q + 6] * inv, o[8 * q + 7] * inv));
        }
      }
    }
  }
  // ---- teardown: the MMA lane saw every product complete; every TMEM access has waited ----
  tc::fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc::fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

template <int D>
int launch(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm, const Params& p, int tokens,
           int q_heads, int batch, cudaStream_t stream) {
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(prefill_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem<D>::kTotal) !=
        cudaSuccess)
      return FB_ERR_LAUNCH;
    configured[dev] = true;
  }
  const int q_tiles = (tokens + kTile - 1) / kTile;
  return launch_ex(prefill_kernel<D>, dim3((q_tiles + 1) / 2, q_heads, batch), dim3(kThreads), Smem<D>::kTotal,
                   stream, 1, qm, km, vm, p);
}

}  // namespace prefill
}  // namespace fb

using namespace fb;

extern "C" int fb_prefill_attention(const void* q, const void* k, const void* v, void* out, int batch, int tokens,
                                    int q_heads, int kv_heads, int head_dim, int capacity, float scale, void* stream) {
  if (!q || !k || !v || !out || batch <= 0 || tokens <= 0 || q_heads <= 0 || kv_heads <= 0) return FB_ERR_ARG;
  if ((head_dim != 64 && head_dim != 128) || q_heads % kv_heads != 0) return FB_ERR_SHAPE;
  if (capacity < tokens || batch > 65535 || q_heads > 65535) return FB_ERR_SHAPE;
  if (static_cast<long long>(batch) * kv_heads * capacity >= (1ll << 31) ||
      static_cast<long long>(batch) * q_heads * tokens >= (1ll << 31))
    return FB_ERR_SHAPE;
  prefill::Params p{};
  p.out = static_cast<__nv_bfloat16*>(out);
  p.batch = batch;
  p.tokens = tokens;
  p.q_heads = q_heads;
  p.kv_heads = kv_heads;
  p.groups = q_heads / kv_heads;
  p.capacity = capacity;
  p.scale_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634);
  p.err = error_word();
  CUtensorMap qm, km, vm;
  int st = encode_bf16_2d(&qm, q, static_cast<uint64_t>(batch) * q_heads * tokens, head_dim, head_dim, 64,
                          prefill::kTile, true);
  if (st != FB_OK) return st;
  const uint64_t kv_rows = static_cast<uint64_t>(batch) * kv_heads * capacity;
  st = encode_bf16_2d(&km, k, kv_rows, head_dim, head_dim, 64, prefill::kTile, true);
  if (st != FB_OK) return st;
  st = encode_bf16_2d(&vm, v, kv_rows, head_dim, head_dim, 64, prefill::kTile, true);
  if (st != FB_OK) return st;
  cudaStream_t stream_ = static_cast<cudaStream_t>(stream);
  return head_dim == 128 ? prefill::launch<128>(qm, km, vm, p, tokens, q_heads, batch, stream_)
                         : prefill::launch<64>(qm, km, vm, p, tokens, q_heads, batch, stream_);
}

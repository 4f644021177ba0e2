// Causal GQA prefill attention (flash attention forward) on the 5th-generation tensor cores
// (sm_100a).
//
// Replaces the reference's prefill path, engine/attention.py:8-21 (`grouped_sdpa` with no
// mask: torch SDPA's Flash backend, is_causal, enable_gqa): for every query token t of a row
// and query head hq, softmax(q . k_j * scale) over keys j <= t of KV head hq / G, times V,
// with fp32 scores and accumulation and P rounded to bf16 for the value product.
//
// B200 design (one CTA per (128-query tile, query head, row); heavy tiles first):
//  * A TMA lane loads the Q tile once and streams 128-key K and V tiles (128-byte swizzle,
//    no multicast) through a 2-stage ring.
//  * A UMMA lane issues S = Q K^T (M = 128 queries, N = 128 keys, K = D) into one of two TMEM
//    buffers and O += P V (N = 128 dims, K = 128 keys; V read MN-major) into a TMEM
//    accumulator; S of tile j+1 runs while the softmax warps work on tile j.
//  * Eight softmax warps, two per query row (64 keys each, exchanging row maxima and sums
//    through spare TMEM columns): row max, P = 2^(s - m) rounded to bf16 into a K-major
//    swizzled tile in shared memory (double-buffered), row sum. The pivot m only moves when a
//    row's max grows by more than 8 (P <= 2^8 otherwise); then the row's O in TMEM is
//    rescaled in place after the previous product completes. Tiles below the diagonal skip
//    the masks.
//  * Every mbarrier wait is bounded; TMEM is freed on every path.
#include "tcgen05.cuh"

namespace fb {
namespace prefill {

constexpr int kTile = 128;      // queries per CTA tile and keys per K/V tile
constexpr int kSoftmaxWarps = 8;  // warp w: query rows 32*(w%4).., key half / O-column half w/4
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 10 * 32;
constexpr int kTmemCols = 512;  // S double buffer (2 x 128) + O (<= 128) + row exchange columns
constexpr int kTmemO = 256;
constexpr int kTmemXchg = 384;  // [parity][half] row maxima, then [half] row sums
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
  static constexpr int kPBytes = 2 * kBox;            // 128 query rows x 128 keys
  static constexpr int kStageBytes = 2 * kTileBytes;  // K then V
  static constexpr int kStages = 2;
  static constexpr int kQOff = 0;
  static constexpr int kStageOff = kTileBytes;
  static constexpr int kPOff = kStageOff + kStages * kStageBytes;  // two P tiles
  static constexpr int kBarOff = kPOff + 2 * kPBytes;
  static constexpr int kBars = 16;
  static constexpr int kTotal = 1024 + kBarOff + kBars * 8 + 16;
  static_assert(kTotal <= 227 * 1024, "prefill shared memory");
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, const Params p) {
  using S = Smem<D>;
  constexpr int kDim = D;
  constexpr uint32_t kIdescS = tc::idesc_bf16(kTile, kTile, false, false);
  constexpr uint32_t kIdescO = tc::idesc_bf16(kTile, D, false, true);
  pdl_wait();
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = base + S::kQOff;
  uint8_t* stages = base + S::kStageOff;
  uint8_t* p_s = base + S::kPOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + S::kBarOff);
  uint64_t* full = bars;        // [2] K/V stage landed
  uint64_t* empty = bars + 2;   // [2] K/V stage consumed (O product done)
  uint64_t* s_full = bars + 4;  // [2] S buffer computed
  uint64_t* s_free = bars + 6;  // [2] S buffer read by the softmax warps
  uint64_t* p_full = bars + 8;  // [2] P tile written
  uint64_t* o_done = bars + 10; // [2] O product of a tile (by P buffer) complete
  uint64_t* q_full = bars + 12;
  uint64_t* done = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q_tiles = (p.tokens + kTile - 1) / kTile;
  const int qt = q_tiles - 1 - static_cast<int>(blockIdx.x);  // the heaviest (latest) tiles first
  const int hq = blockIdx.y, b = blockIdx.z;
  const int hkv = hq / p.groups;
  const int kv_tiles = qt + 1;  // keys [0, 128 * (qt + 1)) cover every query of the tile

  if (warp == kProducerWarp && lane == 0) {
    for (int x = 0; x < 2; ++x) {
      mbar_init(&full[x], 1);
      mbar_init(&empty[x], 1);
      mbar_init(&s_full[x], 1);
      mbar_init(&s_free[x], kSoftmaxWarps);
      mbar_init(&p_full[x], kSoftmaxWarps);  // eight softmax warps arrive on each
      mbar_init(&o_done[x], 1);
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
  const uint32_t tmem_o = tmem + kTmemO;

  if (warp == kProducerWarp) {
    // ============================ TMA producer ============================
    if (lane == 0) {
      const int qrow = (b * p.q_heads + hq) * p.tokens + qt * kTile;
      mbar_arrive_expect_tx(q_full, S::kTileBytes);
#pragma unroll
      for (int bx = 0; bx < D / 64; ++bx) tma_load_2d(q_s + bx * S::kBox, &qmap, q_full, bx * 64, qrow);
      const int kvrow = (b * p.kv_heads + hkv) * p.capacity;
      for (int j = 0; j < kv_tiles && !*abort_flag; ++j) {
        const int st = j & 1;
        if (j >= 2 && !mbar_wait_bounded(&empty[st], ((j - 2) >> 1) & 1)) {
          raise_error(p.err, kErrTimeoutEmpty);
          *abort_flag = 1;
          break;
        }
        uint8_t* kt = stages + st * S::kStageBytes;
        uint8_t* vt = kt + S::kTileBytes;
        mbar_arrive_expect_tx(&full[st], S::kStageBytes);
        const int row = kvrow + j * kTile;
#pragma unroll
        for (int bx = 0; bx < D / 64; ++bx) {
          tma_load_2d(kt + bx * S::kBox, &kmap, &full[st], bx * 64, row);
          tma_load_2d(vt + bx * S::kBox, &vmap, &full[st], bx * 64, row);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ============================ UMMA issuer ============================
    if (lane == 0) {
      const uint32_t q_addr = smem_u32(q_s), p_addr = smem_u32(p_s);
      auto issue_o = [&](int j) -> bool {
        const int x = j & 1;
        if (!mbar_wait_bounded(&p_full[x], (j >> 1) & 1)) return false;
        tc::fence_after();
        const uint32_t v_addr = smem_u32(stages + x * S::kStageBytes + S::kTileBytes);
        const uint32_t pb = p_addr + x * S::kPBytes;
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk) {
          const uint32_t off_p = (kk >> 2) * S::kBox + (kk & 3) * 32;  // 16 keys of the P rows
          const uint32_t off_v = kk * 16 * 128;                          // 16 key rows of V
          tc::mma_bf16(tmem_o, tc::desc_sw128(pb + off_p, 16, 1024), tc::desc_sw128(v_addr + off_v, S::kBox, 1024),
                       kIdescO, (j > 0 || kk > 0) ? 1u : 0u);
        }
        tc::commit(&o_done[x]);
        tc::commit(&empty[x]);  // both products of tile j have read its K/V stage
        return true;
      };
      bool ok = mbar_wait_bounded(q_full, 0);
      for (int j = 0; j < kv_tiles && ok; ++j) {
        const int x = j & 1;
        ok = mbar_wait_bounded(&full[x], (j >> 1) & 1) && (j < 2 || mbar_wait_bounded(&s_free[x], ((j - 2) >> 1) & 1));
        if (!ok || *abort_flag) break;
        tc::fence_after();
        const uint32_t k_addr = smem_u32(stages + x * S::kStageBytes);
#pragma unroll
        for (int kk = 0; kk < kDim / 16; ++kk) {
          const uint32_t off = (kk >> 2) * S::kBox + (kk & 3) * 32;  // 16 dims of the 128-byte rows
          tc::mma_bf16(tmem + 128 * x, tc::desc_sw128(q_addr + off, 16, 1024), tc::desc_sw128(k_addr + off, 16, 1024),
                       kIdescS, kk > 0 ? 1u : 0u);
        }
        tc::commit(&s_full[x]);
        if (j >= 1) ok = issue_o(j - 1);
      }
      if (ok && !*abort_flag) ok = issue_o(kv_tiles - 1);
      if (!ok) {
        raise_error(p.err, kErrTimeoutMma);
        *abort_flag = 1;
      }
      tc::commit(done);  // arrives once every product issued above has completed
      if (!mbar_wait_bounded(done, 0)) raise_error(p.err, kErrTimeoutDrain);
    }
    __syncwarp();
  } else {
    // ============================ softmax warps ============================
    // Warp w reads TMEM lanes 32*(w%4).. (its query rows) and key columns [64h, 64h + 64) of S,
    // h = w / 4, and owns O columns [h*D/2, (h+1)*D/2). The two warps of a row exchange their
    // partial row maxima (and, at the end, row sums) through spare TMEM columns and a named
    // barrier per warp pair; both then take identical pivot decisions. Control flow stays
    // warp-uniform: tcgen05.ld/st are .sync.aligned.
    const int quarter = warp & 3, half = warp >> 2;
    const int row = quarter * 32 + lane;  // query row of the tile = TMEM lane
    const int t = qt * kTile + row;       // its token
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t pair_bar = 1 + quarter;  // named barriers 1..4, 64 threads each
    const float sl2 = p.scale_log2;
    const int last_key = min(t, p.tokens - 1);  // keys <= last_key are visible to this row
    float pivot = -INFINITY, lsum = 0.f;
    bool ok = true;
    for (int j = 0; j < kv_tiles; ++j) {
      const int x = j & 1;
      const bool waited = !*abort_flag && mbar_wait_bounded(&s_full[x], (j >> 1) & 1);
      if (!__all_sync(0xffffffffu, waited)) {
        ok = false;
        break;
      }
      tc::fence_after();
      const uint32_t s_addr = tmem + 128 * x + 64 * half + lane_base;
      const int key0 = j * kTile + 64 * half;  // this warp's first key
      // a tile below the diagonal is visible to every query row of this tile
      const bool interior = j < qt;
      // this warp's 64 scores of the row, read from TMEM once and kept for the P pass
      float sv[64];
      {
        float* lo = sv;
        float* hi = sv + 32;
        tc::ld32(s_addr, *reinterpret_cast<float(*)[32]>(lo));
        tc::ld32(s_addr + 32, *reinterpret_cast<float(*)[32]>(hi));
      }
      // S_x is free for the score product of tile j + 2 as soon as both halves are read
      tc::fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[x]);
      // raw maximum, scaled once: sl2 > 0 and rounding is monotone, so max(s) * sl2 equals
      // max(s * sl2). Interior tiles take the mask-free path.
      float mx = -INFINITY;
      if (interior) {
#pragma unroll
        for (int c = 0; c < 64; ++c) mx = fmaxf(mx, sv[c]);
      } else {
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (key0 + c <= last_key) mx = fmaxf(mx, sv[c]);
      }
      if (mx != -INFINITY) mx *= sl2;
      // the row's other half: exchange partial maxima through TMEM column [parity][half]
      tc::st1(tmem + kTmemXchg + 2 * x + half + lane_base, mx);
      tc::fence_before();
      asm volatile("bar.sync %0, 64;" ::"r"(pair_bar) : "memory");
      tc::fence_after();
      mx = fmaxf(mx, tc::ld1(tmem + kTmemXchg + 2 * x + (1 - half) + lane_base));
      // lazy rescale: a row's pivot moves only when its max exceeds the pivot by more than 8
      float corr = 1.f;
      const bool need = mx > pivot + kRescaleAbove || (pivot == -INFINITY && mx > -INFINITY);
      if (need) {
        corr = pivot == -INFINITY ? 0.f : tc::ex2_approx(pivot - mx);
        pivot = mx;
      }
      lsum *= corr;
      // P tile x was last read by the product of tile j - 2
      if (j >= 2) {
        const bool free = mbar_wait_bounded(&o_done[x], ((j - 2) >> 1) & 1);
        if (!__all_sync(0xffffffffu, free)) {
          ok = false;
          break;
        }
      }
      const float piv = pivot == -INFINITY ? 0.f : pivot;
      // this warp's 64 keys are box `half` of the K-major P tile
      uint8_t* pt = p_s + x * S::kPBytes + half * S::kBox;
#pragma unroll
      for (int c0 = 0; c0 < 64; c0 += 32) {
        const float* v = sv + c0;
        uint32_t packed[16];
        if (interior) {
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const float p0 = tc::ex2_approx(fmaf(v[c], sl2, -piv));
            const float p1 = tc::ex2_approx(fmaf(v[c + 1], sl2, -piv));
            lsum += p0 + p1;
            packed[c / 2] = pack_bf16x2(p0, p1);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const bool see0 = key0 + c0 + c <= last_key;
            const bool see1 = key0 + c0 + c + 1 <= last_key;
            const float p0 = see0 ? tc::ex2_approx(fmaf(v[c], sl2, -piv)) : 0.f;
            const float p1 = see1 ? tc::ex2_approx(fmaf(v[c + 1], sl2, -piv)) : 0.f;
            lsum += p0 + p1;
            packed[c / 2] = pack_bf16x2(p0, p1);
          }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(pt + sw128(row, (c0 >> 3) + q)) =
              make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
      }
      // O rescale after the P pass (the scores are dead by then): the product of tile j - 1 must
      // have landed, and the product of tile j waits for p_full below
      if (j >= 1 && __any_sync(0xffffffffu, need)) {
        // the previous tile's product must have landed in O before this warp's half of the
        // rows' O is rescaled (rows that keep their pivot multiply by 1)
        const bool landed = mbar_wait_bounded(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1);
        if (!__all_sync(0xffffffffu, landed)) {
          ok = false;
          break;
        }
        tc::fence_after();
#pragma unroll
        for (int c0 = 0; c0 < kDim / 2; c0 += 32) {
          float o[32];
          tc::ld32(tmem_o + half * (kDim / 2) + lane_base + c0, o);
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] *= corr;
          tc::st32(tmem_o + half * (kDim / 2) + lane_base + c0, o);
        }
      }
      // V rows past the prompt: zeroed so stale cache values never meet a zero weight
      if (half == 0 && j * kTile + kTile > p.tokens && j * kTile + row >= p.tokens) {
        uint8_t* vt = stages + x * S::kStageBytes + S::kTileBytes;
#pragma unroll
        for (int bx = 0; bx < D / 64; ++bx)
#pragma unroll
          for (int c16 = 0; c16 < 8; ++c16)
            *reinterpret_cast<uint4*>(vt + bx * S::kBox + row * 128 + c16 * 16) = make_uint4(0, 0, 0, 0);
      }
      tc::fence_before();        // the rescaled O (TMEM) before the product of tile j
      fence_proxy_async_smem();  // P and zeroed V rows (shared memory) before the product
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[x]);
    }
    if (ok) {
      const bool landed = mbar_wait_bounded(&o_done[(kv_tiles - 1) & 1], ((kv_tiles - 1) >> 1) & 1);
      ok = __all_sync(0xffffffffu, landed);
    }
    if (!ok) {
      raise_error(p.err, kErrTimeoutMma);
      *abort_flag = 1;
    }
    if (ok) {
      // row sum = both halves' partial sums (TMEM exchange, column [half] past the maxima)
      tc::fence_after();
      tc::st1(tmem + kTmemXchg + 4 + half + lane_base, lsum);
      tc::fence_before();
      asm volatile("bar.sync %0, 64;" ::"r"(pair_bar) : "memory");
      tc::fence_after();
      const float total = lsum + tc::ld1(tmem + kTmemXchg + 4 + (1 - half) + lane_base);
      const float inv = total > 0.f ? 1.f / total : 0.f;
      // every lane reads its O row half (uniform TMEM loads); rows past the prompt are not stored
      __nv_bfloat16* dst =
          p.out + ((static_cast<size_t>(b) * p.tokens + t) * p.q_heads + hq) * kDim + half * (kDim / 2);
#pragma unroll
      for (int c0 = 0; c0 < kDim / 2; c0 += 32) {
        float o[32];
        tc::ld32(tmem_o + half * (kDim / 2) + lane_base + c0, o);
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
  return launch_ex(prefill_kernel<D>, dim3(q_tiles, q_heads, batch), dim3(kThreads), Smem<D>::kTotal, stream, 1, qm,
                   km, vm, p);
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

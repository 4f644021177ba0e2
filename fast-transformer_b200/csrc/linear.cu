// Skinny bf16 projection y[M, N] = x[M, K] @ W[N, K]^T for decode (M <= 64), sm_100a.
//
// Same contract as the reference's skinny kinds (engine/kernels/linear.py:27-93,
// gemm.py:51-425): fp32 accumulation and one rounding to bf16 per output; split-K fp32
// partials may be handed to a consumer that sums them in split order (merged.py:13-45).
//
// The weight stream is the whole cost (HBM-bound: every weight byte is read once per step):
//  * Grid = (N / 128 tiles) x S K-splits, two CTAs per SM; S (fb_linear_splits) fills whole
//    waves of the machine. One producer lane TMA-loads 128x64 weight tiles (L2 evict-first)
//    and the matching M x 64 slab of x (rows past M zero-filled by the tensor map) into a
//    6-stage mbarrier ring of 128-byte-swizzled buffers; four consumer warps each own 32 output
//    features and run mma.sync m16n8k16 with x as the 16-row A operand.
//  * Launched with programmatic stream serialization: the producer issues the weight stages
//    before griddepcontrol.wait, so the stream overlaps the previous kernel's tail; nothing an
//    earlier kernel wrote is read before the wait.
//  * Epilogues: fp32 split partials [S, M, N]; or a finished tile - bf16, fp32, SwiGLU on
//    weights packed as 64-row gate/up blocks, or per-row argmax candidates.
//  * Finished tiles with S > 1 (S <= 8) run as a (1, S) thread-block cluster whose CTAs sum
//    the S partials through distributed shared memory, in split order (the bits a split
//    consumer produces). The decode step itself hands split partials to consumer kernels,
//    which measured faster inside the captured step than any in-launch split sum.
#include "common.cuh"

namespace fb {
namespace lin {

constexpr int kTileN = 128;
constexpr int kTileK = 64;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kStages = 6;
constexpr int kMaxTiles = 65535;       // grid x
constexpr int kMaxClusterSplits = 8;  // portable cluster size: K-splits of one finished tile

enum Epilogue : int { kBf16 = 0, kFp32 = 1, kSwiGLU = 2, kSplits = 3, kArgmax = 4 };

struct Params {
  void* out;
  int m, n, k, splits, epilogue;
  long long index_base;  // kArgmax: vocabulary index of column 0
  unsigned* err;
};

template <int MT>
struct Smem {
  static constexpr int MP = MT * 16;
  static constexpr int kWBytes = kTileN * 128;
  static constexpr int kXBytes = MP * 128;
  static constexpr int kStageBytes = kWBytes + kXBytes;
  static constexpr int kTileVals = MP * kTileN * 4;  // staged in the drained stage buffers
  static_assert(kTileVals <= kStages * kStageBytes, "tile values must fit the stage ring");
  static constexpr int kTotal = 1024 + kStages * kStageBytes + 2 * kStages * 8 + 64;
};

__device__ __forceinline__ float silu_bf16(float g) {
  // engine/kernels/swiglu.py:21: SiLU computed in fp32 and rounded to bf16
  return bf16_round(g / (1.0f + expf(-g)));
}

// Column groups (4 fp32 columns) of a tile owned by cluster rank r of S: group cg, or for
// SwiGLU the feature group cg % 16 (gate columns and the matching up columns together).
__device__ __forceinline__ bool owned(int cg, int epi, int r, int S) {
  return ((epi == kSwiGLU ? (cg & 15) : cg) % S) == r;
}

// Epilogue over a finished tile held in shared memory (vals[MP][128], fp32), for the column
// groups this CTA owns (all of them when the tile was not split).
template <int MT>
__device__ void epilogue(const Params& p, const float* vals, int tile, int tid, int r, int S) {
  constexpr int MP = MT * 16;
  const int n0 = tile * kTileN;
  if (p.epilogue == kArgmax) {
    // Each row's (max, first index) over this tile's bf16-rounded logits (the values the
    // projection would store), packed as index << 32 | value bits into cand[m][tile]. The
    // tile's accumulation is one split over the whole of K, like the projection at S = 1.
    const int warp = tid >> 5, lane = tid & 31;
    for (int m = warp; m < p.m; m += kConsumerWarps) {
      const float4 v4 = *reinterpret_cast<const float4*>(vals + m * kTileN + lane * 4);
      const float vs[4] = {v4.x, v4.y, v4.z, v4.w};
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = n0 + lane * 4 + e;
        const float v = bf16_round(vs[e]);
        if (col < p.n && (v > bv || (v == bv && col < bi))) {
          bv = v;
          bi = col;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (lane == 0) {
        // no candidate (all -inf or NaN): index sentinel 0x7fffffff, never offset
        const uint32_t index = bi == 0x7fffffff ? 0x7fffffffu : static_cast<uint32_t>(p.index_base + bi);
        static_cast<uint64_t*>(p.out)[static_cast<size_t>(m) * gridDim.x + tile] =
            (static_cast<uint64_t>(index) << 32) | __float_as_uint(bv);
      }
    }
    return;
  }
  if (p.epilogue == kSwiGLU) {
    // Tile rows [0, 64) are gate features f0..f0+63 and rows [64, 128) the up features of the
    // same f: out[m][f] = bf16(bf16(silu(bf16(g))) * bf16(u)).
    const int f0 = tile * (kTileN / 2);
    const int width = p.n / 2;
    for (int e = tid; e < p.m * (kTileN / 2); e += kConsumerWarps * 32) {
      const int m = e / (kTileN / 2), j = e % (kTileN / 2);
      if (f0 + j >= width || !owned(j >> 2, kSwiGLU, r, S)) continue;
      const float g = bf16_round(vals[m * kTileN + j]);
      const float u = bf16_round(vals[m * kTileN + 64 + j]);
      static_cast<__nv_bfloat16*>(p.out)[static_cast<size_t>(m) * width + f0 + j] =
          __float2bfloat16_rn(silu_bf16(g) * u);
    }
    return;
  }
  for (int e = tid; e < p.m * (kTileN / 4); e += kConsumerWarps * 32) {
    const int m = e / (kTileN / 4), c4 = e % (kTileN / 4);
    const int col = n0 + c4 * 4;
    if (col >= p.n || !owned(c4, p.epilogue, r, S)) continue;
    const float4 v = *reinterpret_cast<const float4*>(vals + m * kTileN + c4 * 4);
    if (p.epilogue == kFp32) {
      *reinterpret_cast<float4*>(static_cast<float*>(p.out) + static_cast<size_t>(m) * p.n + col) = v;
    } else {
      uint2 w;
      w.x = pack_bf16x2(v.x, v.y);
      w.y = pack_bf16x2(v.z, v.w);
      *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.out) + static_cast<size_t>(m) * p.n + col) = w;
    }
  }
  (void)MP;
}

template <int MT>
__global__ void __launch_bounds__(kThreads)
    linear_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                  const __grid_constant__ Params p) {
  using S = Smem<MT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  float* vals = reinterpret_cast<float*>(base);  // reused once the ring has drained
  uint64_t* full = reinterpret_cast<uint64_t*>(base + kStages * S::kStageBytes);
  uint64_t* empty = full + kStages;
  volatile int* flags = reinterpret_cast<volatile int*>(empty + kStages);  // [0] abort

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int n0 = tile * kTileN;
  const int chunks = (p.k + kTileK - 1) / kTileK;
  const int c0 = static_cast<int>((static_cast<long long>(chunks) * split) / p.splits);
  const int c1 = static_cast<int>((static_cast<long long>(chunks) * (split + 1)) / p.splits);
  const int count = c1 - c0;
  // finished-tile epilogues reduce the K-splits of a tile across its cluster (dims 1 x S)
  const bool clustered = p.epilogue != kSplits && p.splits > 1;

  if (warp == kConsumerWarps && lane == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_barrier_init();
    prefetch_tensormap(&xmap);
    prefetch_tensormap(&wmap);
    flags[0] = 0;
  }
  __syncthreads();
  pdl_trigger();

  if (warp == kConsumerWarps) {
    if (lane == 0) {
      const uint64_t evict_first = l2_evict_first_policy();
      // Weights do not depend on the previous kernel: fill the ring before waiting on it.
      const int pre = count < kStages ? count : kStages;
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], S::kStageBytes);
        tma_load_2d_hint(base + i * S::kStageBytes, &wmap, &full[i], (c0 + i) * kTileK, n0, evict_first);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i)
        tma_load_2d(base + i * S::kStageBytes + S::kWBytes, &xmap, &full[i], (c0 + i) * kTileK, 0);
      for (int i = pre; i < count; ++i) {
        const int s = i % kStages;
        if (flags[0]) break;
        if (!mbar_wait_bounded(&empty[s], ((i / kStages) - 1) & 1)) {
          raise_error(p.err, kErrTimeoutEmpty);
          flags[0] = 1;
          break;
        }
        uint8_t* wt = base + s * S::kStageBytes;
        mbar_arrive_expect_tx(&full[s], S::kStageBytes);
        tma_load_2d_hint(wt, &wmap, &full[s], (c0 + i) * kTileK, n0, evict_first);
        tma_load_2d(wt + S::kWBytes, &xmap, &full[s], (c0 + i) * kTileK, 0);
      }
    }
    __syncwarp();
    if (clustered) {
      // every thread of every CTA in the cluster takes the same two cluster barriers
      cluster_sync();
      cluster_sync();
    }
    return;
  }

  pdl_wait();  // outputs may be read by the previous kernel
  const int g = lane >> 2, c4 = lane & 3;
  const int tid = threadIdx.x;
  const int q = lane >> 3;
  const int a_row = (lane & 7) + (q & 1) * 8, a_kc = q >> 1;
  const int b_row = (lane & 7) + (q >> 1) * 8, b_kc = q & 1;
  float acc[MT][4][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) acc[mt][nt][0] = acc[mt][nt][1] = acc[mt][nt][2] = acc[mt][nt][3] = 0.f;
  bool aborted = false;
  for (int i = 0; i < count; ++i) {
    const int s = i % kStages;
    if (!mbar_wait_bounded(&full[s], (i / kStages) & 1)) {
      raise_error(p.err, kErrTimeoutFull);
      flags[0] = 1;
    }
    if (flags[0]) {
      aborted = true;  // still takes the cluster barriers below
      break;
    }
    const uint32_t wt = smem_u32(base + s * S::kStageBytes);
    const uint32_t xt = wt + S::kWBytes;
#pragma unroll
    for (int ks = 0; ks < kTileK / 16; ++ks) {
      uint32_t a[MT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
        ldmatrix_x4(xt + sw128(mt * 16 + a_row, ks * 2 + a_kc), a[mt][0], a[mt][1], a[mt][2], a[mt][3]);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(wt + sw128(warp * 32 + np * 16 + b_row, ks * 2 + b_kc), b0, b1, b2, b3);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          mma_bf16_16816(acc[mt][np * 2 + 0], a[mt][0], a[mt][1], a[mt][2], a[mt][3], b0, b1);
          mma_bf16_16816(acc[mt][np * 2 + 1], a[mt][0], a[mt][1], a[mt][2], a[mt][3], b2, b3);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  if (aborted && !clustered) return;

  if (p.epilogue == kSplits) {
    // fp32 partials [S, M, N]: C fragment rows (g, g+8), columns (2c, 2c+1) of each 16x8 tile
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int col = n0 + warp * 32 + nt * 8 + 2 * c4;
        if (col >= p.n) continue;
#pragma unroll
        for (int hlf = 0; hlf < 2; ++hlf) {
          const int row = mt * 16 + g + hlf * 8;
          if (row >= p.m) continue;
          float* dst = static_cast<float*>(p.out) + (static_cast<size_t>(split) * p.m + row) * p.n + col;
          *reinterpret_cast<float2*>(dst) = make_float2(acc[mt][nt][hlf * 2], acc[mt][nt][hlf * 2 + 1]);
        }
      }
    return;
  }

  // ---- finished-tile epilogues: this split's sums -> shared tile (the ring has drained) ----
  asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int col = warp * 32 + nt * 8 + 2 * c4;
      *reinterpret_cast<float2*>(vals + (mt * 16 + g) * kTileN + col) = make_float2(acc[mt][nt][0], acc[mt][nt][1]);
      *reinterpret_cast<float2*>(vals + (mt * 16 + g + 8) * kTileN + col) = make_float2(acc[mt][nt][2], acc[mt][nt][3]);
    }
  if (!clustered) {
    asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
    epilogue<MT>(p, vals, tile, tid, 0, 1);
    return;
  }
  // Split tile: sum the S partials through distributed shared memory. Rank r sums the column
  // groups it owns over ranks 0..S-1 in order (deterministic) into its own tile, then runs
  // the epilogue for those groups.
  cluster_sync();  // every CTA's partial tile is complete and visible cluster-wide
  const int r = static_cast<int>(cluster_rank());
  const int nsplit = p.splits;
  if (!aborted) {
    const uint32_t local = smem_u32(vals);
    for (int e = tid; e < p.m * (kTileN / 4); e += kConsumerWarps * 32) {
      const int m = e / (kTileN / 4), cg = e % (kTileN / 4);
      if (!owned(cg, p.epilogue, r, nsplit)) continue;
      const uint32_t off = static_cast<uint32_t>((m * kTileN + cg * 4) * 4);
      float4 parts[8];
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (q < nsplit) parts[q] = ld_cluster_f4(map_shared(local + off, q));
      float4 sum = parts[0];
#pragma unroll
      for (int q = 1; q < 8; ++q)
        if (q < nsplit) {
          sum.x += parts[q].x;
          sum.y += parts[q].y;
          sum.z += parts[q].z;
          sum.w += parts[q].w;
        }
      *reinterpret_cast<float4*>(vals + m * kTileN + cg * 4) = sum;
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
    epilogue<MT>(p, vals, tile, tid, r, nsplit);
  }
  cluster_sync();  // no CTA leaves while another may still read its tile
}

template <int MT>
int launch(const CUtensorMap& xm, const CUtensorMap& wm, const Params& p, cudaStream_t stream) {
  using S = Smem<MT>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(linear_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal) !=
        cudaSuccess)
      return FB_ERR_LAUNCH;
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.n + kTileN - 1) / kTileN, p.splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = S::kTotal;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (p.epilogue != kSplits && p.splits > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = p.splits;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  if (cudaLaunchKernelEx(&cfg, linear_kernel<MT>, xm, wm, p) != cudaSuccess) return FB_ERR_LAUNCH;
  return check_launch();
}

int row_tiles(int m) { return m <= 16 ? 1 : m <= 32 ? 2 : 4; }

int ctas_per_sm(int mt) {
  const int total = mt == 1 ? Smem<1>::kTotal : mt == 2 ? Smem<2>::kTotal : Smem<4>::kTotal;
  int per = (227 * 1024) / (total + 1024);
  return per < 1 ? 1 : per;
}

}  // namespace lin
}  // namespace fb

using namespace fb;

extern "C" int fb_linear_splits(int m, int n, int k) {
  if (m <= 0 || n <= 0 || k <= 0) return 1;
  const int tiles = (n + lin::kTileN - 1) / lin::kTileN;
  const int chunks = (k + lin::kTileK - 1) / lin::kTileK;
  const int slots = sm_count() * lin::ctas_per_sm(lin::row_tiles(m));
  // One wave: the most splits whose CTAs are all resident at once (a second, partial wave
  // costs more than the extra streams gain), keeping at least 4 chunks per CTA so each
  // pipeline fills. Measured on B200 at M=16: N=4096/K=4096 -> 9 (7.3 us), N=6144 -> 6
  // (9.3 us), N=24576 -> 1 (36 us); every other S was slower or within noise.
  int best = tiles >= slots ? 1 : slots / tiles;
  if (best > chunks / 4) best = chunks / 4;
  return best < 1 ? 1 : best;
}

extern "C" int fb_linear_finished_splits(int m, int n, int k) {
  // fb_linear_splits capped by the thread-block cluster that sums a finished tile's splits
  const int s = fb_linear_splits(m, n, k);
  if (s <= 1) return 1;
  return s < lin::kMaxClusterSplits ? s : lin::kMaxClusterSplits;
}

static int linear_impl(const void* x, const void* w, void* out, int m, int n, int k, int epilogue, int splits,
                       void* stream, int64_t index_base = 0) {
  if (!x || !w || !out || m <= 0 || n <= 0 || k <= 0 || splits <= 0) return FB_ERR_ARG;
  if (m > 64 || k % 8 != 0 || n % 8 != 0) return FB_ERR_SHAPE;
  if ((n + lin::kTileN - 1) / lin::kTileN > lin::kMaxTiles) return FB_ERR_SHAPE;
  if (epilogue == lin::kSwiGLU && n % lin::kTileN != 0) return FB_ERR_SHAPE;
  if (epilogue == lin::kArgmax && splits != 1) return FB_ERR_SHAPE;
  if (splits > (k + lin::kTileK - 1) / lin::kTileK || splits > 65535) return FB_ERR_SHAPE;
  if (epilogue != lin::kSplits && splits > lin::kMaxClusterSplits) return FB_ERR_SHAPE;
  const int mt = lin::row_tiles(m);
  CUtensorMap xm, wm;
  int st = encode_bf16_2d(&xm, x, m, k, k, 64, mt * 16, true);
  if (st != FB_OK) return st;
  st = encode_bf16_2d(&wm, w, n, k, k, 64, lin::kTileN, true);
  if (st != FB_OK) return st;
  lin::Params p{};
  p.out = out;
  p.m = m;
  p.n = n;
  p.k = k;
  p.splits = splits;
  p.epilogue = epilogue;
  p.index_base = index_base;
  p.err = error_word();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (mt == 1) return lin::launch<1>(xm, wm, p, s);
  if (mt == 2) return lin::launch<2>(xm, wm, p, s);
  return lin::launch<4>(xm, wm, p, s);
}

extern "C" int fb_linear(const void* x, const void* w, void* out, int m, int n, int k, int epilogue, int splits,
                         void* stream) {
  if (epilogue < lin::kBf16 || epilogue > lin::kSplits) return FB_ERR_ARG;
  return linear_impl(x, w, out, m, n, k, epilogue, splits, stream);
}

extern "C" size_t fb_argmax_candidates_bytes(int m, int n) {
  if (m <= 0 || n <= 0) return 0;
  return static_cast<size_t>(m) * ((n + lin::kTileN - 1) / lin::kTileN) * sizeof(uint64_t);
}

extern "C" int fb_linear_argmax(const void* x, const void* w, int m, int n, int k, int64_t index_base, void* cand,
                                void* stream) {
  if (!cand || index_base < 0 || index_base + n > 0x7ffffffe) return FB_ERR_ARG;
  return linear_impl(x, w, cand, m, n, k, lin::kArgmax, 1, stream, index_base);
}

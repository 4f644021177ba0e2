// Skinny bf16 projection y[M, N] = x[M, K] @ W[N, K]^T for decode (M <= 64), sm_100a.
//
// Same contract as the reference's skinny kinds (engine/kernels/linear.py:27-93,
// gemm.py:51-425): fp32 accumulation, one rounding to bf16, optional split-K fp32
// partials [S, M, N] that a consumer sums in split order (merged.py:13-45).
//
// The weight stream is the whole cost (HBM-bound: every weight byte is read once per
// step), so the kernel is a TMA pipeline: one producer lane loads 128x64 weight tiles
// and the matching Mx64 slab of x (rows past M are zero-filled by the tensor map) into
// an NS-stage ring of 128-byte-swizzled buffers; four consumer warps each own 32 output
// features and run mma.sync m16n8k16 with x as the 16-row A operand and W rows as B.
// Grid = (N / 128 tiles) x (K splits); the split count is chosen on the host so that the
// grid fills whole waves of the machine.
#include "common.cuh"

namespace fb {
namespace lin {

constexpr int kTileN = 128;
constexpr int kTileK = 64;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kStages = 6;

struct Params {
  void* out;
  int m, n, k, splits, out_fp32;
  unsigned* err;
};

template <int MT>
struct Smem {
  static constexpr int kWBytes = kTileN * 128;
  static constexpr int kXBytes = MT * 16 * 128;
  static constexpr int kStageBytes = kWBytes + kXBytes;
  static constexpr int kTotal = 1024 + kStages * kStageBytes + 2 * kStages * 8 + 16;
};

template <int MT>
__global__ void __launch_bounds__(kThreads)
    linear_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                  const Params p) {
  using S = Smem<MT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(base + kStages * S::kStageBytes);
  uint64_t* empty = full + kStages;
  volatile int* abort_flag = reinterpret_cast<int*>(empty + kStages);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kTileN;
  const int split = blockIdx.y;
  const int chunks = (p.k + kTileK - 1) / kTileK;
  const int c0 = static_cast<int>((static_cast<long long>(chunks) * split) / p.splits);
  const int c1 = static_cast<int>((static_cast<long long>(chunks) * (split + 1)) / p.splits);
  const int count = c1 - c0;

  if (warp == kConsumerWarps && lane == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_barrier_init();
    prefetch_tensormap(&xmap);
    prefetch_tensormap(&wmap);
    *abort_flag = 0;
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    if (lane == 0) {
      const uint64_t evict_first = l2_evict_first_policy();
      for (int i = 0; i < count; ++i) {
        const int s = i % kStages;
        if (*abort_flag) break;
        if (i >= kStages && !mbar_wait_bounded(&empty[s], ((i / kStages) - 1) & 1)) {
          raise_error(p.err, kErrTimeoutEmpty);
          *abort_flag = 1;
          break;
        }
        uint8_t* wt = base + s * S::kStageBytes;
        uint8_t* xt = wt + S::kWBytes;
        mbar_arrive_expect_tx(&full[s], S::kStageBytes);
        const int kx = (c0 + i) * kTileK;
        tma_load_2d_hint(wt, &wmap, &full[s], kx, n0, evict_first);
        tma_load_2d(xt, &xmap, &full[s], kx, 0);
      }
    }
    return;
  }

  const int g = lane >> 2, c = lane & 3;
  float acc[MT][4][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) acc[mt][nt][0] = acc[mt][nt][1] = acc[mt][nt][2] = acc[mt][nt][3] = 0.f;

  // ldmatrix lane roles
  const int q = lane >> 3;  // matrix index within an x4 load
  // A (x): matrices (rows 0-7,k0-7) (rows 8-15,k0-7) (rows 0-7,k8-15) (rows 8-15,k8-15)
  const int a_row = (lane & 7) + (q & 1) * 8;
  const int a_kc = q >> 1;
  // B (W): matrices (n 0-7,k0-7) (n 0-7,k8-15) (n 8-15,k0-7) (n 8-15,k8-15)
  const int b_row = (lane & 7) + (q >> 1) * 8;
  const int b_kc = q & 1;

  for (int i = 0; i < count; ++i) {
    const int s = i % kStages;
    if (!mbar_wait_bounded(&full[s], (i / kStages) & 1)) {
      raise_error(p.err, kErrTimeoutFull);
      *abort_flag = 1;
      break;
    }
    if (*abort_flag) break;
    const uint32_t wt = smem_u32(base + s * S::kStageBytes);
    const uint32_t xt = wt + S::kWBytes;
#pragma unroll
    for (int ks = 0; ks < kTileK / 16; ++ks) {
      uint32_t a[MT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
        ldmatrix_x4(xt + sw128(mt * 16 + a_row, ks * 2 + a_kc), a[mt][0], a[mt][1], a[mt][2],
                    a[mt][3]);
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

  // Epilogue: C fragment rows (g, g+8) x cols (2c, 2c+1) of each 16x8 tile.
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int col = n0 + warp * 32 + nt * 8 + 2 * c;
      if (col >= p.n) continue;
#pragma unroll
      for (int hlf = 0; hlf < 2; ++hlf) {
        const int row = mt * 16 + g + hlf * 8;
        if (row >= p.m) continue;
        const float v0 = acc[mt][nt][hlf * 2 + 0], v1 = acc[mt][nt][hlf * 2 + 1];
        if (p.splits == 1 && !p.out_fp32) {
          *reinterpret_cast<uint32_t*>(static_cast<__nv_bfloat16*>(p.out) +
                                       static_cast<size_t>(row) * p.n + col) = pack_bf16x2(v0, v1);
        } else {
          float* dst = static_cast<float*>(p.out) +
                       (static_cast<size_t>(split) * p.m + row) * p.n + col;
          *reinterpret_cast<float2*>(dst) = make_float2(v0, v1);
        }
      }
    }
  }
}

template <int MT>
int launch(const CUtensorMap& xm, const CUtensorMap& wm, const Params& p, cudaStream_t stream) {
  using S = Smem<MT>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(linear_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             S::kTotal) != cudaSuccess)
      return FB_ERR_LAUNCH;
    configured[dev] = true;
  }
  dim3 grid((p.n + kTileN - 1) / kTileN, p.splits);
  linear_kernel<MT><<<grid, kThreads, S::kTotal, stream>>>(xm, wm, p);
  return check_launch();
}

}  // namespace lin
}  // namespace fb

using namespace fb;

extern "C" int fb_linear_splits(int m, int n, int k) {
  if (m <= 0 || n <= 0 || k <= 0) return 1;
  const int tiles = (n + lin::kTileN - 1) / lin::kTileN;
  const int chunks = (k + lin::kTileK - 1) / lin::kTileK;
  const int mt = m <= 16 ? 1 : m <= 32 ? 2 : 4;
  const int stage = lin::kTileN * 128 + mt * 16 * 128;
  const int per_sm = (227 * 1024) / (1024 + lin::kStages * stage + 128);
  const int slots = sm_count() * (per_sm > 0 ? per_sm : 1);
  // Modelled time ~ waves * (chunks per CTA + fixed ramp of ~2 chunks); pick the best S
  // with at least 4 chunks per CTA so the pipeline fills.
  int best = 1;
  double best_cost = 1e30;
  for (int s = 1; s <= 32; ++s) {
    if (chunks / s < 4 && s > 1) break;
    const int ctas = tiles * s;
    const int waves = (ctas + slots - 1) / slots;
    const double per_cta = static_cast<double>(chunks) / s + 2.0;
    const double cost = waves * per_cta + (s > 1 ? 0.02 * s * m : 0.0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

extern "C" int fb_linear(const void* x, const void* w, void* out, int m, int n, int k, int splits,
                         int out_fp32, void* stream) {
  if (!x || !w || !out || m <= 0 || n <= 0 || k <= 0 || splits <= 0) return FB_ERR_ARG;
  if (m > 64 || k % 8 != 0 || n % 8 != 0) return FB_ERR_SHAPE;
  const int chunks = (k + lin::kTileK - 1) / lin::kTileK;
  if (splits > chunks) return FB_ERR_SHAPE;
  const int mt = m <= 16 ? 1 : m <= 32 ? 2 : 4;
  CUtensorMap xm, wm;
  int st = encode_bf16_2d(&xm, x, m, k, k, 64, mt * 16, true);
  if (st != FB_OK) return st;
  st = encode_bf16_2d(&wm, w, n, k, k, 64, lin::kTileN, true);
  if (st != FB_OK) return st;
  lin::Params p;
  p.out = out;
  p.m = m;
  p.n = n;
  p.k = k;
  p.splits = splits;
  p.out_fp32 = out_fp32;
  p.err = error_word();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (mt == 1) return lin::launch<1>(xm, wm, p, s);
  if (mt == 2) return lin::launch<2>(xm, wm, p, s);
  return lin::launch<4>(xm, wm, p, s);
}

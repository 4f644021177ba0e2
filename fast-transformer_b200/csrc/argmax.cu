// First-index argmax over bf16 logits (sm_100a): torch.argmax's answer in two launches.
//
// Same two-stage structure and tie rule as the reference (engine/kernels/argmax.py:19-48):
// stage one reduces each (row, 8192-column block) to its maximum and the lowest index of
// that maximum; stage two picks each row's first best block. bf16 -> fp32 is exact, so the
// comparison order gives exactly the lowest index of the row maximum.
#include "common.cuh"

namespace fb {
namespace amax {

constexpr int kBlock = 8192;  // columns per stage-one CTA (argmax.py:51 block=8192)
constexpr int kThreads = 256;

__device__ __forceinline__ void better(float& v, int& i, float ov, int oi) {
  // larger value wins; equal values -> lower index
  if (ov > v || (ov == v && oi < i)) {
    v = ov;
    i = oi;
  }
}

__global__ void __launch_bounds__(kThreads)
    block_argmax_kernel(const __nv_bfloat16* logits, int64_t vocab, int blocks, float* best_value,
                        int* best_index) {
  __shared__ float sv[kThreads / 32];
  __shared__ int si[kThreads / 32];
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.y;
  const int blk = blockIdx.x;
  const int64_t c0 = static_cast<int64_t>(blk) * kBlock;
  const __nv_bfloat16* src = logits + static_cast<int64_t>(row) * vocab;
  float v = -INFINITY;
  int idx = 0x7fffffff;
  // Each thread scans 8-column groups; groups are visited in ascending order per thread.
  const bool aligned = (vocab % 8 == 0);
  for (int grp = threadIdx.x; grp < kBlock / 8; grp += kThreads) {
    const int64_t col = c0 + grp * 8;
    if (col >= vocab) break;
    if (aligned) {
      const uint4 w = *reinterpret_cast<const uint4*>(src + col);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        better(v, idx, bf16_lo(ws[e]), static_cast<int>(col + 2 * e));
        better(v, idx, bf16_hi(ws[e]), static_cast<int>(col + 2 * e + 1));
      }
    } else {
      for (int e = 0; e < 8 && col + e < vocab; ++e)
        better(v, idx, __bfloat162float(src[col + e]), static_cast<int>(col + e));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    better(v, idx, ov, oi);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = v;
    si[warp] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float bv = sv[0];
    int bi = si[0];
    for (int w = 1; w < kThreads / 32; ++w) better(bv, bi, sv[w], si[w]);
    best_value[static_cast<int64_t>(row) * blocks + blk] = bv;
    best_index[static_cast<int64_t>(row) * blocks + blk] = bi;
  }
}

__global__ void __launch_bounds__(32)
    first_best_kernel(const float* best_value, const int* best_index, int blocks, int64_t* out,
                      float* top) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  float v = -INFINITY;
  int idx = 0x7fffffff;
  for (int b = threadIdx.x; b < blocks; b += 32)
    better(v, idx, best_value[static_cast<int64_t>(row) * blocks + b],
           best_index[static_cast<int64_t>(row) * blocks + b]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    better(v, idx, ov, oi);
  }
  if (threadIdx.x == 0) {
    // All -inf (or NaN-only) rows keep index 0, like torch.argmax on an all -inf row.
    out[row] = idx == 0x7fffffff ? 0 : idx;
    if (top != nullptr) top[row] = v;
  }
}

// Per-row reduction of the fused projection's tile candidates (fb_linear_argmax), then, in
// tensor parallelism, the exchange of every rank's best: each rank stores its (value, index)
// as two flagged words (low half the payload, high half (uint32)(*epoch) + 1) into slot
// [row][rank] of every rank's exchange buffer and reduces the world slots once their flags
// match. Every rank applies the same rule to the same words, so all ranks pick the same id.
constexpr int kCandThreads = 128;
constexpr int kMaxWorld = 8;

struct CandParams {
  const uint64_t* cand;  // [rows, tiles]: index << 32 | value bits
  int rows, tiles, world, rank;
  uint64_t* peers[kMaxWorld];  // every rank's exchange buffer, uint64 [rows, world, 2]
  const uint64_t* local;       // this rank's exchange buffer
  const int64_t* epoch;
  int64_t* out;
  float* top;
  unsigned* err;
};

__device__ __forceinline__ void unpack(uint64_t w, float& v, int& i) {
  v = __uint_as_float(static_cast<uint32_t>(w));
  i = static_cast<int>(static_cast<uint32_t>(w >> 32));
}

__global__ void __launch_bounds__(kCandThreads) candidates_kernel(const CandParams p) {
  __shared__ float sv[kCandThreads / 32];
  __shared__ int si[kCandThreads / 32];
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  float v = -INFINITY;
  int idx = 0x7fffffff;
  for (int t = threadIdx.x; t < p.tiles; t += kCandThreads) {
    float ov;
    int oi;
    unpack(p.cand[static_cast<size_t>(row) * p.tiles + t], ov, oi);
    better(v, idx, ov, oi);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    better(v, idx, ov, oi);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = v;
    si[warp] = idx;
  }
  __syncthreads();
  if (warp != 0) return;
  v = sv[0];
  idx = si[0];
  for (int w = 1; w < kCandThreads / 32; ++w) better(v, idx, sv[w], si[w]);
  if (p.world > 1) {
    const uint64_t flag = static_cast<uint64_t>(static_cast<uint32_t>(*p.epoch) + 1u) << 32;
    const size_t mine = (static_cast<size_t>(row) * p.world + p.rank) * 2;
    if (lane < p.world) {
      const uint64_t w0 = flag | __float_as_uint(v), w1 = flag | static_cast<uint32_t>(idx);
      asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p.peers[lane] + mine), "l"(w0), "l"(w1)
                   : "memory");
    }
    v = -INFINITY;
    idx = 0x7fffffff;
    if (lane < p.world) {
      const uint64_t* slot = p.local + (static_cast<size_t>(row) * p.world + lane) * 2;
      const unsigned long long start = globaltimer();
      bool good = p.err == nullptr || (*reinterpret_cast<volatile unsigned*>(p.err) & kErrTimeoutFull) == 0;
      while (good) {
        uint64_t w0, w1;
        asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(slot) : "memory");
        if ((w0 >> 32) == (flag >> 32) && (w1 >> 32) == (flag >> 32)) {
          v = __uint_as_float(static_cast<uint32_t>(w0));
          idx = static_cast<int>(static_cast<uint32_t>(w1));
          break;
        }
        if (globaltimer() - start > kWaitBudgetNs) {
          raise_error(p.err, kErrTimeoutFull);
          good = false;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      better(v, idx, ov, oi);
    }
  }
  if (lane == 0) {
    // All -inf (or NaN-only) rows keep index 0, like torch.argmax on an all -inf row.
    p.out[row] = idx == 0x7fffffff ? 0 : idx;
    if (p.top != nullptr) p.top[row] = v;
  }
}

}  // namespace amax
}  // namespace fb

using namespace fb;

extern "C" size_t fb_argmax_workspace(int rows, int64_t vocab) {
  if (rows <= 0 || vocab <= 0) return 0;
  const int64_t blocks = (vocab + amax::kBlock - 1) / amax::kBlock;
  return static_cast<size_t>(rows) * blocks * (sizeof(float) + sizeof(int)) + 256;
}

extern "C" int fb_argmax(const void* logits, int rows, int64_t vocab, int64_t* out, float* top,
                         void* workspace, size_t workspace_bytes, void* stream) {
  if (!logits || !out || !workspace || rows <= 0 || vocab <= 0) return FB_ERR_ARG;
  if (vocab >= (1ll << 31) || rows > 65535) return FB_ERR_SHAPE;
  if (workspace_bytes < fb_argmax_workspace(rows, vocab)) return FB_ERR_WORKSPACE;
  const int blocks = static_cast<int>((vocab + amax::kBlock - 1) / amax::kBlock);
  float* bv = static_cast<float*>(workspace);
  int* bi = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) +
                                   ((static_cast<size_t>(rows) * blocks * sizeof(float) + 255) &
                                    ~size_t(255)));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool aligned_ptr = (reinterpret_cast<uintptr_t>(logits) & 15u) == 0;
  if (!aligned_ptr) return FB_ERR_ARG;
  int st = launch_ex(amax::block_argmax_kernel, dim3(blocks, rows), dim3(amax::kThreads), 0, s, 1,
                     static_cast<const __nv_bfloat16*>(logits), vocab, blocks, bv, bi);
  if (st != FB_OK) return st;
  return launch_ex(amax::first_best_kernel, dim3(rows), dim3(32), 0, s, 1, bv, bi, blocks, out, top);
}

extern "C" int fb_argmax_candidates(const void* cand, int rows, int tiles, int world, int rank,
                                    void* const* peer_exchange, const void* exchange_local, const int64_t* epoch,
                                    int64_t* out, float* top, void* stream) {
  if (!cand || !out || rows <= 0 || tiles <= 0) return FB_ERR_ARG;
  if (world < 1 || world > amax::kMaxWorld || rank < 0 || rank >= world) return FB_ERR_ARG;
  amax::CandParams p{};
  p.cand = static_cast<const uint64_t*>(cand);
  p.rows = rows;
  p.tiles = tiles;
  p.world = world;
  p.rank = rank;
  if (world > 1) {
    if (!peer_exchange || !exchange_local || !epoch) return FB_ERR_ARG;
    for (int r = 0; r < world; ++r) {
      if (!peer_exchange[r] || (reinterpret_cast<uintptr_t>(peer_exchange[r]) & 15u)) return FB_ERR_ARG;
      p.peers[r] = static_cast<uint64_t*>(peer_exchange[r]);
    }
    p.local = static_cast<const uint64_t*>(exchange_local);
    p.epoch = epoch;
  }
  p.out = out;
  p.top = top;
  p.err = error_word();
  return launch_ex(amax::candidates_kernel, dim3(rows), dim3(amax::kCandThreads), 0, static_cast<cudaStream_t>(stream),
                   1, p);
}

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

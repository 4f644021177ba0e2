// RMSNorm family, SwiGLU and the split-K merge (sm_100a). All HBM/latency bound; one
// CTA per row with 16-byte vector accesses. Cast points follow the reference:
//   rms_norm       engine/kernels/rmsnorm.py:21-46   y = bf16(bf16(x*inv) * w)
//   add_rms_norm   engine/kernels/rmsnorm.py:75-95   s = bf16(x+r); y = bf16(bf16(s*inv) * w)
//   embed_rms_norm engine/kernels/rmsnorm.py:128-142 h = table[id]; y = rms_norm(h)
//   swiglu         engine/kernels/swiglu.py:13-24    y = bf16(bf16(g/(1+exp(-g))) * u)
//   merge          engine/kernels/linear.py:81-93    y = bf16(sum_s partial[s])
// inv = 1/sqrt(mean(x^2) + eps) in fp32. Split-K fp32 inputs are summed in split order
// and rounded to bf16 before use (engine/kernels/merged.py:37-45).
#include "common.cuh"

namespace fb {
namespace norm {

constexpr int kThreads = 256;

// 8 consecutive logical bf16 values starting at element `off` of a tensor that is either
// bf16 (splits == 0) or fp32 split partials [splits, count] (splits >= 1).
__device__ __forceinline__ void load8(const void* src, int splits, size_t count, size_t off,
                                      float (&x)[8]) {
  if (splits == 0) {
    const uint4 w = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(src) + off);
    x[0] = bf16_lo(w.x);
    x[1] = bf16_hi(w.x);
    x[2] = bf16_lo(w.y);
    x[3] = bf16_hi(w.y);
    x[4] = bf16_lo(w.z);
    x[5] = bf16_hi(w.z);
    x[6] = bf16_lo(w.w);
    x[7] = bf16_hi(w.w);
    return;
  }
  const float* f = static_cast<const float*>(src) + off;
  const float4 a = *reinterpret_cast<const float4*>(f);
  const float4 b = *reinterpret_cast<const float4*>(f + 4);
  x[0] = a.x;
  x[1] = a.y;
  x[2] = a.z;
  x[3] = a.w;
  x[4] = b.x;
  x[5] = b.y;
  x[6] = b.z;
  x[7] = b.w;
  // Issue the loads of up to four slabs before adding them (in split order), so a
  // multi-split input costs ceil((S-1)/4) memory round trips rather than S-1.
  for (int s0 = 1; s0 < splits; s0 += 4) {
    float4 c[4], d[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (s0 + j < splits) {
        c[j] = __ldg(reinterpret_cast<const float4*>(f + (s0 + j) * count));
        d[j] = __ldg(reinterpret_cast<const float4*>(f + (s0 + j) * count + 4));
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (s0 + j < splits) {
        x[0] += c[j].x;
        x[1] += c[j].y;
        x[2] += c[j].z;
        x[3] += c[j].w;
        x[4] += d[j].x;
        x[5] += d[j].y;
        x[6] += d[j].z;
        x[7] += d[j].w;
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) x[e] = bf16_round(x[e]);
}

__device__ __forceinline__ void store8(__nv_bfloat16* dst, const float (&y)[8]) {
  uint4 w;
  w.x = pack_bf16x2(y[0], y[1]);
  w.y = pack_bf16x2(y[2], y[3]);
  w.z = pack_bf16x2(y[4], y[5]);
  w.w = pack_bf16x2(y[6], y[7]);
  *reinterpret_cast<uint4*>(dst) = w;
}

__device__ __forceinline__ void load_w8(const __nv_bfloat16* w, int col, float (&x)[8]) {
  const uint4 v = *reinterpret_cast<const uint4*>(w + col);
  x[0] = bf16_lo(v.x);
  x[1] = bf16_hi(v.x);
  x[2] = bf16_lo(v.y);
  x[3] = bf16_hi(v.y);
  x[4] = bf16_lo(v.z);
  x[5] = bf16_hi(v.z);
  x[6] = bf16_lo(v.w);
  x[7] = bf16_hi(v.w);
}

__device__ __forceinline__ float block_sum(float v, float* scratch) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = 0.f;
  const int nw = blockDim.x >> 5;
  for (int i = 0; i < nw; ++i) t += scratch[i];
  __syncthreads();
  return t;
}

// Per-thread register cache: up to kMaxChunks 8-wide chunks per thread (W <= 16384).
constexpr int kMaxChunks = 8;

// mode 0: rms_norm(x)  mode 1: add_rms_norm(x, residual)  mode 2: embed + rms_norm
struct Params {
  const void* x;
  int splits;
  int64_t row_stride;
  const __nv_bfloat16* residual;
  const __nv_bfloat16* w;
  __nv_bfloat16* y;
  __nv_bfloat16* sum;
  const int64_t* ids;
  int64_t vocab;
  int rows, width;
  float eps;
  unsigned* err;
};

template <int MODE>
__global__ void __launch_bounds__(kThreads) rmsnorm_kernel(const Params p) {
  __shared__ float scratch[kThreads / 32];
  const int row = blockIdx.x;
  const int chunks = p.width / 8;
  float v[kMaxChunks][8];
  const void* src = p.x;
  size_t base = static_cast<size_t>(row) * p.width;
  if (MODE == 0) base = static_cast<size_t>(row) * p.row_stride;
  if (MODE == 2) {
    const long long id = p.ids[row];
    if (id < 0 || id >= p.vocab) {
      if (threadIdx.x == 0) raise_error(p.err, kErrBadShape);
      return;
    }
    base = static_cast<size_t>(id) * p.width;
  }
  const size_t count = static_cast<size_t>(p.rows) * p.width;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int ch = threadIdx.x + i * kThreads;
    if (ch < chunks) {
      load8(src, MODE == 1 ? p.splits : 0, count, base + ch * 8, v[i]);
      if (MODE == 1) {
        float r[8];
        load8(p.residual, 0, 0, static_cast<size_t>(row) * p.width + ch * 8, r);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[i][e] = bf16_round(v[i][e] + r[e]);
        store8(p.sum + static_cast<size_t>(row) * p.width + ch * 8, v[i]);
      }
      if (MODE == 2) store8(p.sum + static_cast<size_t>(row) * p.width + ch * 8, v[i]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[i][e] * v[i][e];
    }
  }
  ss = block_sum(ss, scratch);
  const float inv = 1.0f / sqrtf(ss / static_cast<float>(p.width) + p.eps);
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int ch = threadIdx.x + i * kThreads;
    if (ch < chunks) {
      float w[8], y[8];
      load_w8(p.w, ch * 8, w);
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = bf16_round(v[i][e] * inv) * w[e];
      const size_t out = (MODE == 0 ? static_cast<size_t>(row) * p.row_stride
                                    : static_cast<size_t>(row) * p.width) +
                         ch * 8;
      store8(p.y + out, y);
    }
  }
}

__global__ void __launch_bounds__(kThreads)
    swiglu_kernel(const void* packed, int splits, __nv_bfloat16* out, int rows, int width) {
  const int64_t flat = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const int per_row = width / 8;
  if (flat >= static_cast<int64_t>(rows) * per_row) return;
  const int row = static_cast<int>(flat / per_row);
  const int ch = static_cast<int>(flat % per_row);
  const size_t count = static_cast<size_t>(rows) * 2 * width;
  const size_t base = static_cast<size_t>(row) * 2 * width + ch * 8;
  float g[8], u[8], y[8];
  load8(packed, splits, count, base, g);
  load8(packed, splits, count, base + width, u);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float act = bf16_round(g[e] / (1.0f + expf(-g[e])));
    y[e] = act * u[e];
  }
  store8(out + static_cast<size_t>(row) * width + ch * 8, y);
}

__global__ void __launch_bounds__(kThreads)
    merge_kernel(const float* partial, int splits, int64_t count, void* out, int out_fp32) {
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) * 4;
  if (i >= count) return;
  float x[4];
  const int n = count - i < 4 ? static_cast<int>(count - i) : 4;
  for (int e = 0; e < n; ++e) x[e] = partial[i + e];
  for (int s0 = 1; s0 < splits; s0 += 4) {
    float y[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      for (int e = 0; e < n; ++e) y[j][e] = s0 + j < splits ? partial[(s0 + j) * count + i + e] : 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (s0 + j < splits)
        for (int e = 0; e < n; ++e) x[e] += y[j][e];
  }
  if (out_fp32) {
    for (int e = 0; e < n; ++e) static_cast<float*>(out)[i + e] = x[e];
  } else {
    for (int e = 0; e < n; ++e) static_cast<__nv_bfloat16*>(out)[i + e] = __float2bfloat16_rn(x[e]);
  }
}

// Tensor-parallel all-reduce consumer fused with the residual add + RMSNorm. Every rank's
// projection kernel pushed its fp32 [rows, W] partial into slab `rank` of this rank's
// recv[use] and added one arrival per 128-column tile to arrivals[use]; once all
// world * tiles arrivals are in, the slabs are summed in rank order (identical bits on every
// rank), rounded to bf16 (the projection's output) and fed to add_rms_norm's arithmetic.
// The last CTA to finish resets the use's arrival and completion counters for the next step.
struct ReduceParams {
  const float* recv;        // [uses, world, rows, W] on this rank
  unsigned* arrivals;       // [uses] on this rank, bumped by every rank's producer
  unsigned* done;           // [uses] on this rank
  int use, world, expected;
  const __nv_bfloat16* residual;
  const __nv_bfloat16* w;
  __nv_bfloat16* out;
  __nv_bfloat16* sum;
  int rows, width;
  float eps;
  unsigned* err;
};

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kThreads) allreduce_add_rmsnorm_kernel(const ReduceParams p) {
  __shared__ float scratch[kThreads / 32];
  __shared__ int ok;
  const int row = blockIdx.x;
  if (threadIdx.x == 0) {
    const unsigned long long start = globaltimer();
    // After one wait has given up, fail fast instead of spending the budget again per use.
    int good = p.err == nullptr || (*reinterpret_cast<volatile unsigned*>(p.err) & kErrTimeoutFull) == 0;
    while (good && ld_acquire_sys(p.arrivals + p.use) < static_cast<unsigned>(p.expected)) {
      if (globaltimer() - start > kWaitBudgetNs) {
        raise_error(p.err, kErrTimeoutFull);
        good = 0;
        break;
      }
    }
    ok = good;
  }
  __syncthreads();
  const int chunks = p.width / 8;
  const size_t slab = static_cast<size_t>(p.rows) * p.width;
  const float* recv = p.recv + static_cast<size_t>(p.use) * p.world * slab + static_cast<size_t>(row) * p.width;
  float v[kMaxChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int ch = threadIdx.x + i * kThreads;
    if (ch < chunks && ok) {
      float x[8];
      // rank-order fp32 sum of the partials, then the projection's bf16 rounding
      load8(recv, p.world, slab, static_cast<size_t>(ch) * 8, x);
      float r[8];
      load8(p.residual, 0, 0, static_cast<size_t>(row) * p.width + ch * 8, r);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[i][e] = bf16_round(x[e] + r[e]);
      store8(p.sum + static_cast<size_t>(row) * p.width + ch * 8, v[i]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[i][e] * v[i][e];
    }
  }
  ss = block_sum(ss, scratch);
  const float inv = 1.0f / sqrtf(ss / static_cast<float>(p.width) + p.eps);
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int ch = threadIdx.x + i * kThreads;
    if (ch < chunks && ok) {
      float w[8], y[8];
      load_w8(p.w, ch * 8, w);
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = bf16_round(v[i][e] * inv) * w[e];
      store8(p.out + static_cast<size_t>(row) * p.width + ch * 8, y);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(p.done + p.use, 1u) == static_cast<unsigned>(gridDim.x) - 1) {
      // every row has read this use's slabs: ready for the next step
      p.done[p.use] = 0;
      atomicExch(p.arrivals + p.use, 0u);
    }
  }
}

int check_width(int width) {
  if (width <= 0 || width % 8 != 0) return FB_ERR_SHAPE;
  if (width > 8 * kThreads * kMaxChunks) return FB_ERR_SHAPE;
  return FB_OK;
}

}  // namespace norm
}  // namespace fb

using namespace fb;

extern "C" int fb_rmsnorm(const void* x, int64_t row_stride, const void* w, void* y, int rows,
                          int width, float eps, void* stream) {
  if (!x || !w || !y || rows <= 0 || row_stride < width) return FB_ERR_ARG;
  int st = norm::check_width(width);
  if (st != FB_OK) return st;
  if (row_stride % 8 != 0) return FB_ERR_SHAPE;
  norm::Params p{};
  p.x = x;
  p.splits = 0;
  p.row_stride = row_stride;
  p.w = static_cast<const __nv_bfloat16*>(w);
  p.y = static_cast<__nv_bfloat16*>(y);
  p.rows = rows;
  p.width = width;
  p.eps = eps;
  p.err = error_word();
  norm::rmsnorm_kernel<0><<<rows, norm::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch();
}

extern "C" int fb_add_rmsnorm(const void* x, int x_splits, const void* residual, const void* w,
                              void* out, void* sum, int rows, int width, float eps, void* stream) {
  if (!x || !residual || !w || !out || !sum || rows <= 0 || x_splits < 0) return FB_ERR_ARG;
  int st = norm::check_width(width);
  if (st != FB_OK) return st;
  norm::Params p{};
  p.x = x;
  p.splits = x_splits;
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.w = static_cast<const __nv_bfloat16*>(w);
  p.y = static_cast<__nv_bfloat16*>(out);
  p.sum = static_cast<__nv_bfloat16*>(sum);
  p.rows = rows;
  p.width = width;
  p.eps = eps;
  p.err = error_word();
  norm::rmsnorm_kernel<1><<<rows, norm::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch();
}

extern "C" int fb_embed_rmsnorm(const int64_t* ids, const void* table, int64_t vocab, const void* w,
                                void* y, void* hidden, int rows, int width, float eps,
                                void* stream) {
  if (!ids || !table || !w || !y || !hidden || rows <= 0 || vocab <= 0) return FB_ERR_ARG;
  int st = norm::check_width(width);
  if (st != FB_OK) return st;
  norm::Params p{};
  p.x = table;
  p.splits = 0;
  p.w = static_cast<const __nv_bfloat16*>(w);
  p.y = static_cast<__nv_bfloat16*>(y);
  p.sum = static_cast<__nv_bfloat16*>(hidden);
  p.ids = ids;
  p.vocab = vocab;
  p.rows = rows;
  p.width = width;
  p.eps = eps;
  p.err = error_word();
  norm::rmsnorm_kernel<2><<<rows, norm::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch();
}

extern "C" int fb_swiglu(const void* packed, int splits, void* out, int rows, int width,
                         void* stream) {
  if (!packed || !out || rows <= 0 || splits < 0 || width <= 0) return FB_ERR_ARG;
  if (width % 8 != 0) return FB_ERR_SHAPE;
  const int64_t threads = static_cast<int64_t>(rows) * (width / 8);
  const int64_t blocks = (threads + norm::kThreads - 1) / norm::kThreads;
  if (blocks >= (1ll << 31)) return FB_ERR_SHAPE;
  norm::swiglu_kernel<<<static_cast<unsigned>(blocks), norm::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      packed, splits, static_cast<__nv_bfloat16*>(out), rows, width);
  return check_launch();
}

extern "C" int fb_merge_splits(const void* partial, int splits, int64_t count, void* out,
                               int out_fp32, void* stream) {
  if (!partial || !out || splits <= 0 || count <= 0) return FB_ERR_ARG;
  const int64_t threads = (count + 3) / 4;
  const int blocks = static_cast<int>((threads + norm::kThreads - 1) / norm::kThreads);
  norm::merge_kernel<<<blocks, norm::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const float*>(partial), splits, count, out, out_fp32);
  return check_launch();
}

extern "C" int fb_allreduce_add_rmsnorm(const void* recv, void* arrivals, void* done, int use, int world,
                                        int expected, const void* residual, const void* w, void* out, void* sum,
                                        int rows, int width, float eps, void* stream) {
  if (!recv || !arrivals || !done || !residual || !w || !out || !sum) return FB_ERR_ARG;
  if (use < 0 || world < 1 || expected < 1 || rows <= 0) return FB_ERR_ARG;
  int st = norm::check_width(width);
  if (st != FB_OK) return st;
  norm::ReduceParams p;
  p.recv = static_cast<const float*>(recv);
  p.arrivals = static_cast<unsigned*>(arrivals);
  p.done = static_cast<unsigned*>(done);
  p.use = use;
  p.world = world;
  p.expected = expected;
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.w = static_cast<const __nv_bfloat16*>(w);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.sum = static_cast<__nv_bfloat16*>(sum);
  p.rows = rows;
  p.width = width;
  p.eps = eps;
  p.err = error_word();
  norm::allreduce_add_rmsnorm_kernel<<<rows, norm::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch();
}

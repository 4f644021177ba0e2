// RMSNorm family, SwiGLU and the split-K merge (sm_100a). All HBM/latency bound, 16-byte
// vector accesses; an RMSNorm row is spread over a thread-block cluster at decode sizes. Cast points follow the reference:
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

constexpr int kThreads = 256;     // elementwise kernels (swiglu, merge)
constexpr int kMaxThreads = 256;  // RMSNorm CTAs
constexpr int kMaxPer = 4;        // 8-wide chunks per RMSNorm thread
constexpr int kMaxCluster = 8;    // CTAs sharing one RMSNorm row
constexpr int kSlabBatch = 8;     // split slabs whose loads are in flight together
constexpr int kMaxWorld = 8;      // tensor-parallel ranks summed by mode 3

// 8 consecutive logical bf16 values starting at element `off` of a tensor that is either
// bf16 (splits == 0) or fp32 split partials [splits, slab] (splits >= 1). Up to eight slabs
// are loaded before they are added (in split order), so S <= 8 costs one memory round trip.
__device__ __forceinline__ void sum8_fp32(const float* f, int splits, size_t slab, float (&x)[8]);

__device__ __forceinline__ void load8(const void* src, int splits, size_t slab, size_t off,
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
  sum8_fp32(static_cast<const float*>(src) + off, splits, slab, x);
#pragma unroll
  for (int e = 0; e < 8; ++e) x[e] = bf16_round(x[e]);
}

// The fp32 sum, in split order, of 8 consecutive values of `splits` slabs (no rounding).
__device__ __forceinline__ void sum8_fp32(const float* f, int splits, size_t slab, float (&x)[8]) {
  for (int s0 = 0; s0 < splits; s0 += kSlabBatch) {
    float4 c[kSlabBatch], d[kSlabBatch];
#pragma unroll
    for (int j = 0; j < kSlabBatch; ++j) {
      if (s0 + j < splits) {
        c[j] = __ldcg(reinterpret_cast<const float4*>(f + (s0 + j) * slab));
        d[j] = __ldcg(reinterpret_cast<const float4*>(f + (s0 + j) * slab + 4));
      }
    }
#pragma unroll
    for (int j = 0; j < kSlabBatch; ++j) {
      if (s0 + j == 0) {
        x[0] = c[0].x;
        x[1] = c[0].y;
        x[2] = c[0].z;
        x[3] = c[0].w;
        x[4] = d[0].x;
        x[5] = d[0].y;
        x[6] = d[0].z;
        x[7] = d[0].w;
      } else if (s0 + j < splits) {
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
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(w + col));
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

// Mode 3 input: 8 consecutive values of each of `world` slabs of flagged words (low half the
// fp32 bits, high half the flag), summed in rank order and rounded to bf16 once every word
// carries `flag`. Polls with all slabs' loads in flight; gives up after the wait budget (or
// at once if an earlier wait already gave up) and returns false.
__device__ __forceinline__ bool load8_flagged(const uint64_t* src, int world, size_t slab, uint32_t flag,
                                              unsigned* err, float (&x)[8]) {
  unsigned long long start = 0;
  for (;;) {
    bool ready = true;
    // two passes of four ranks keep 32 words in flight per thread
#pragma unroll
    for (int q0 = 0; q0 < kMaxWorld; q0 += 4) {
      uint64_t w[4][8];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (q0 + j < world) {
          const uint64_t* s = src + (q0 + j) * slab;
#pragma unroll
          for (int i = 0; i < 4; ++i)
            asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];"
                         : "=l"(w[j][2 * i]), "=l"(w[j][2 * i + 1])
                         : "l"(s + 2 * i));
        }
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (q0 + j < world) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            ready = ready && static_cast<uint32_t>(w[j][e] >> 32) == flag;
            const float v = __uint_as_float(static_cast<uint32_t>(w[j][e]));
            x[e] = q0 + j == 0 ? v : x[e] + v;
          }
        }
    }
    if (ready) break;
    if (start == 0) start = globaltimer();
    if ((err != nullptr && (*reinterpret_cast<volatile unsigned*>(err) & kErrTimeoutFull) != 0) ||
        globaltimer() - start > kWaitBudgetNs) {
      raise_error(err, kErrTimeoutFull);
      return false;
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) x[e] = bf16_round(x[e]);
  return true;
}

// mode 0: rms_norm(x)          mode 1: add_rms_norm(x, residual)
// mode 2: embed + rms_norm     mode 3: tensor-parallel all-reduce + add_rms_norm
//
// Mode 3: every rank pushed its fp32 [rows, W] partial, as flagged words, into slab `rank` of
// this rank's receive buffer (fb_allreduce_push); once every word carries this step's flag the
// slabs are summed in rank order (identical bits on every rank), rounded to bf16 (the
// projection's output) and fed to add_rms_norm's arithmetic.
struct Params {
  const void* x;          // mode 3: this use's receive slabs, uint64 words [world, rows, W]
  int splits;             // fp32 slabs in x (0: x is bf16); mode 3: world
  int64_t row_stride;     // mode 0
  const __nv_bfloat16* residual;
  const __nv_bfloat16* w;
  __nv_bfloat16* y;
  __nv_bfloat16* sum;
  const int64_t* ids;     // mode 2
  int64_t vocab;
  const int64_t* epoch;   // mode 3: the flag is (uint32)(*epoch) + 1
  int rows, width;
  float eps;
  unsigned* err;
};

// Grid: rows * C CTAs, clusters of C (C = gridDim.x / rows) along x; CTA `rank` of a row's
// cluster owns chunks [rank * per, (rank + 1) * per) of the row (8 values per chunk), each
// thread up to kMaxPer of them. The row's sum of squares is reduced per CTA, then across
// the cluster through distributed shared memory in rank order (the same order, hence the
// same bits, in every CTA).
template <int MODE>
__global__ void __launch_bounds__(kMaxThreads) rmsnorm_kernel(const Params p) {
  __shared__ float scratch[kMaxThreads / 32];
  __shared__ float cluster_ss[kMaxCluster];  // every CTA's sum of squares, by cluster rank
  const int C = gridDim.x / p.rows;
  const int row = blockIdx.x / C;
  const int rank = blockIdx.x % C;
  const int chunks = p.width / 8;
  const int per = (chunks + C - 1) / C;
  const int c0 = rank * per;
  const int c1 = min(chunks, c0 + per);
  const int T = blockDim.x;
  // the gains are never written while decoding: load them before the dependency wait
  float wv[kMaxPer][8];
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int ch = c0 + threadIdx.x + i * T;
    if (ch < c1) load_w8(p.w, ch * 8, wv[i]);
  }
  pdl_wait();
  pdl_trigger();

  const void* src = p.x;
  size_t base = static_cast<size_t>(row) * p.width;
  if (MODE == 0) base = static_cast<size_t>(row) * p.row_stride;
  if (MODE == 2) {
    const long long id = p.ids[row];
    if (id < 0 || id >= p.vocab) {  // the whole cluster (one row) leaves before any barrier
      if (threadIdx.x == 0 && rank == 0) raise_error(p.err, kErrBadShape);
      return;
    }
    base = static_cast<size_t>(id) * p.width;
  }
  const uint32_t flag = MODE == 3 ? static_cast<uint32_t>(*p.epoch) + 1u : 0u;
  const int split_count = (MODE == 1 || MODE == 3) ? p.splits : 0;
  const size_t slab = static_cast<size_t>(p.rows) * p.width;
  // Every CTA of the row's cluster announces that it runs; the wait below, before the first
  // remote shared-memory store, then costs nothing.
  if (C > 1) cluster_arrive_relaxed();
  // The residual's loads are issued with (not after) the input's: it was written before the
  // previous kernel completed.
  float res[kMaxPer][8];
  if (MODE == 1 || MODE == 3) {
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      const int ch = c0 + threadIdx.x + i * T;
      if (ch < c1) load8(p.residual, 0, 0, static_cast<size_t>(row) * p.width + ch * 8, res[i]);
    }
  }
  float v[kMaxPer][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int ch = c0 + threadIdx.x + i * T;
    if (ch < c1) {
      if (MODE == 3) {
        if (!load8_flagged(static_cast<const uint64_t*>(src) + base + ch * 8, p.splits, slab, flag, p.err, v[i]))
#pragma unroll
          for (int e = 0; e < 8; ++e) v[i][e] = 0.f;
      } else {
        load8(src, split_count, slab, base + ch * 8, v[i]);
      }
      if (MODE == 1 || MODE == 3) {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[i][e] = bf16_round(v[i][e] + res[i][e]);
        store8(p.sum + static_cast<size_t>(row) * p.width + ch * 8, v[i]);
      }
      if (MODE == 2) store8(p.sum + static_cast<size_t>(row) * p.width + ch * 8, v[i]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[i][e] * v[i][e];
    }
  }
  ss = block_sum(ss, scratch);
  if (C > 1) {
    // thread q stores this CTA's sum into slot `rank` of cluster CTA q; after the barrier every
    // CTA adds the C slots of its own shared memory in rank order (the same bits everywhere)
    // and nothing reads or writes another CTA's shared memory any more.
    cluster_wait();  // every CTA of the cluster has started
    if (threadIdx.x < C) st_cluster_f32(map_shared(smem_u32(&cluster_ss[rank]), threadIdx.x), ss);
    cluster_sync();
    float total = 0.f;
    for (int q = 0; q < C; ++q) total += cluster_ss[q];
    ss = total;
  }
  const float inv = 1.0f / sqrtf(ss / static_cast<float>(p.width) + p.eps);
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int ch = c0 + threadIdx.x + i * T;
    if (ch < c1) {
      float y[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = bf16_round(v[i][e] * inv) * wv[i][e];
      const size_t out = (MODE == 0 ? static_cast<size_t>(row) * p.row_stride
                                    : static_cast<size_t>(row) * p.width) +
                         ch * 8;
      store8(p.y + out, y);
    }
  }
}

constexpr int kSwigluThreads = 128;

// Four output features per thread: the gate and up values of every split slab are loaded
// together (up to 8 slabs in flight for each), summed in split order and rounded to bf16,
// then bf16(bf16(silu(g)) * u) (engine/kernels/swiglu.py:13-24).
__global__ void __launch_bounds__(kSwigluThreads)
    swiglu_kernel(const void* packed, int splits, __nv_bfloat16* out, int rows, int width, int blocked) {
  pdl_wait();
  pdl_trigger();
  const int64_t flat = static_cast<int64_t>(blockIdx.x) * kSwigluThreads + threadIdx.x;
  const int per_row = width / 4;
  if (flat >= static_cast<int64_t>(rows) * per_row) return;
  const int row = static_cast<int>(flat / per_row);
  const int f = static_cast<int>(flat % per_row) * 4;
  // [gate | up] halves, or 64-column gate/up blocks interleaved (features 64i..64i+63 in
  // columns 128i.. and their up halves in 128i+64..)
  const size_t gate_col = blocked ? static_cast<size_t>(f / 64) * 128 + f % 64 : f;
  const size_t up_col = blocked ? gate_col + 64 : static_cast<size_t>(f) + width;
  const size_t base = static_cast<size_t>(row) * 2 * width;
  float g[4], u[4];
  if (splits == 0) {
    const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(packed) + base;
    const uint2 gw = *reinterpret_cast<const uint2*>(src + gate_col);
    const uint2 uw = *reinterpret_cast<const uint2*>(src + up_col);
    g[0] = bf16_lo(gw.x), g[1] = bf16_hi(gw.x), g[2] = bf16_lo(gw.y), g[3] = bf16_hi(gw.y);
    u[0] = bf16_lo(uw.x), u[1] = bf16_hi(uw.x), u[2] = bf16_lo(uw.y), u[3] = bf16_hi(uw.y);
  } else {
    const float* src = static_cast<const float*>(packed) + base;
    const size_t slab = static_cast<size_t>(rows) * 2 * width;
    for (int s0 = 0; s0 < splits; s0 += kSlabBatch) {
      float4 gs[kSlabBatch], us[kSlabBatch];
#pragma unroll
      for (int j = 0; j < kSlabBatch; ++j)
        if (s0 + j < splits) {
          gs[j] = __ldcg(reinterpret_cast<const float4*>(src + (s0 + j) * slab + gate_col));
          us[j] = __ldcg(reinterpret_cast<const float4*>(src + (s0 + j) * slab + up_col));
        }
#pragma unroll
      for (int j = 0; j < kSlabBatch; ++j) {
        if (s0 + j == 0) {
          g[0] = gs[0].x, g[1] = gs[0].y, g[2] = gs[0].z, g[3] = gs[0].w;
          u[0] = us[0].x, u[1] = us[0].y, u[2] = us[0].z, u[3] = us[0].w;
        } else if (s0 + j < splits) {
          g[0] += gs[j].x, g[1] += gs[j].y, g[2] += gs[j].z, g[3] += gs[j].w;
          u[0] += us[j].x, u[1] += us[j].y, u[2] += us[j].z, u[3] += us[j].w;
        }
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      g[e] = bf16_round(g[e]);
      u[e] = bf16_round(u[e]);
    }
  }
  float y[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) y[e] = bf16_round(g[e] / (1.0f + expf(-g[e]))) * u[e];
  uint2 w;
  w.x = pack_bf16x2(y[0], y[1]);
  w.y = pack_bf16x2(y[2], y[3]);
  *reinterpret_cast<uint2*>(out + static_cast<size_t>(row) * width + f) = w;
}

__global__ void __launch_bounds__(kThreads)
    merge_kernel(const float* partial, int splits, int64_t count, void* out, int out_fp32) {
  pdl_wait();
  pdl_trigger();
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

// Launch shape of the RMSNorm kernel: CTAs per row (cluster size) and threads per CTA.
struct Shape {
  int cluster, threads;
};

int shape_for(int rows, int width, Shape* out) {
  if (width <= 0 || width % 8 != 0) return FB_ERR_SHAPE;
  const int chunks = width / 8;
  // Few rows (decode): spread each row over a cluster so its loads use many SMs. Many rows
  // (prefill): one CTA per row unless the row does not fit one CTA.
  int c = 1;
  if (rows < 2 * sm_count()) c = chunks >= 512 ? 8 : chunks >= 256 ? 4 : chunks >= 128 ? 2 : 1;
  while (c < kMaxCluster && (chunks + c - 1) / c > kMaxThreads * kMaxPer) c *= 2;
  const int per = (chunks + c - 1) / c;
  if (per > kMaxThreads * kMaxPer) return FB_ERR_SHAPE;
  int t = per <= kMaxThreads ? per : (per + kMaxPer - 1) / kMaxPer;
  t = (t + 31) / 32 * 32;
  if (t > kMaxThreads) t = kMaxThreads;
  out->cluster = c;
  out->threads = t;
  return FB_OK;
}

template <int MODE>
int launch_rmsnorm(const Params& p, void* stream) {
  Shape sh;
  const int st = shape_for(p.rows, p.width, &sh);
  if (st != FB_OK) return st;
  const long long grid = static_cast<long long>(p.rows) * sh.cluster;
  if (grid >= (1ll << 31)) return FB_ERR_SHAPE;
  return launch_ex(rmsnorm_kernel<MODE>, dim3(static_cast<unsigned>(grid)), dim3(sh.threads), 0,
                   static_cast<cudaStream_t>(stream), sh.cluster, p);
}

int check_width(int width) {
  Shape sh;
  return shape_for(1, width, &sh);
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
  return norm::launch_rmsnorm<0>(p, stream);
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
  return norm::launch_rmsnorm<1>(p, stream);
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
  return norm::launch_rmsnorm<2>(p, stream);
}

extern "C" int fb_swiglu(const void* packed, int splits, void* out, int rows, int width,
                         void* stream) {
  if (!packed || !out || rows <= 0 || splits < 0 || width <= 0) return FB_ERR_ARG;
  if (width % 8 != 0) return FB_ERR_SHAPE;
  const int64_t threads = static_cast<int64_t>(rows) * (width / 4);
  const int64_t blocks = (threads + norm::kSwigluThreads - 1) / norm::kSwigluThreads;
  if (blocks >= (1ll << 31)) return FB_ERR_SHAPE;
  return launch_ex(norm::swiglu_kernel, dim3(static_cast<unsigned>(blocks)), dim3(norm::kSwigluThreads), 0,
                   static_cast<cudaStream_t>(stream), 1, packed, splits, static_cast<__nv_bfloat16*>(out), rows,
                   width, 0);
}

extern "C" int fb_swiglu_blocked(const void* packed, int splits, void* out, int rows, int width, void* stream) {
  if (!packed || !out || rows <= 0 || splits < 0 || width <= 0) return FB_ERR_ARG;
  if (width % 64 != 0) return FB_ERR_SHAPE;
  const int64_t threads = static_cast<int64_t>(rows) * (width / 4);
  const int64_t blocks = (threads + norm::kSwigluThreads - 1) / norm::kSwigluThreads;
  if (blocks >= (1ll << 31)) return FB_ERR_SHAPE;
  return launch_ex(norm::swiglu_kernel, dim3(static_cast<unsigned>(blocks)), dim3(norm::kSwigluThreads), 0,
                   static_cast<cudaStream_t>(stream), 1, packed, splits, static_cast<__nv_bfloat16*>(out), rows,
                   width, 1);
}

extern "C" int fb_merge_splits(const void* partial, int splits, int64_t count, void* out,
                               int out_fp32, void* stream) {
  if (!partial || !out || splits <= 0 || count <= 0) return FB_ERR_ARG;
  const int64_t threads = (count + 3) / 4;
  const int blocks = static_cast<int>((threads + norm::kThreads - 1) / norm::kThreads);
  return launch_ex(norm::merge_kernel, dim3(blocks), dim3(norm::kThreads), 0, static_cast<cudaStream_t>(stream), 1,
                   static_cast<const float*>(partial), splits, count, out, out_fp32);
}

extern "C" int fb_allreduce_sum_add_rmsnorm(const void* recv, int use, int world, const int64_t* epoch,
                                            const void* residual, const void* w, void* out, void* sum, int rows,
                                            int width, float eps, void* stream) {
  if (!recv || !epoch || !residual || !w || !out || !sum) return FB_ERR_ARG;
  if (use < 0 || world < 1 || world > norm::kMaxWorld || rows <= 0) return FB_ERR_ARG;
  int st = norm::check_width(width);
  if (st != FB_OK) return st;
  const size_t slab = static_cast<size_t>(rows) * width;
  norm::Params p{};
  p.x = static_cast<const uint64_t*>(recv) + static_cast<size_t>(use) * world * slab;
  p.splits = world;
  p.epoch = epoch;
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.w = static_cast<const __nv_bfloat16*>(w);
  p.y = static_cast<__nv_bfloat16*>(out);
  p.sum = static_cast<__nv_bfloat16*>(sum);
  p.rows = rows;
  p.width = width;
  p.eps = eps;
  p.err = error_word();
  return norm::launch_rmsnorm<3>(p, stream);
}

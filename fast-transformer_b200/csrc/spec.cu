// Speculation bookkeeping for exact speculative decoding (sm_100a): the four fused programs of
// the reference's engine/kernels/spec.py, as CUDA kernels with the same semantics.
//
//  propose   (spec.py:16-124)  per row: the newest token's earlier occurrences ranked by how
//            long a suffix agrees (up to `maxlen`), chain drafts copied from the best match
//            (else followed through the successor table), the chain depth chosen by match
//            length, then alternatives to draft 1 (stale hint, other occurrences' followers,
//            successor entries; all distinct from draft 1), chains and RoPE phases.
//  within_margin (spec.py:127-151)  is draft `slot` within `margin` of the winning logit of
//            the row that produced it (relaxed acceptance).
//  settle    (spec.py:169-240)  keep the chain drafts up to the first illegal one or branch to
//            an alternative equal to the model's first choice, clamp at `limit`, emit what was
//            in context into `result` and `history`, plan the KV move, advance `position`.
//  relocate  (spec.py:243-270)  copy one K/V slot per row in every (K/V, layer) plane.
//
// All of it is integer/index work on a few KB per row, latency-bound; every index that comes
// from device data is bounds-checked (the error word records a bad one and the access is
// skipped) rather than trusted.
#include "common.cuh"

namespace fb {
namespace spec {

constexpr int kThreads = 256;
constexpr int kMaxTokens = 64;  // tokens per row (verify block width)
constexpr int kMaxLanes = kMaxTokens;

struct ProposeParams {
  const int64_t* history;  // [B, size]
  int64_t size;
  const int64_t* position;  // [B]
  const int64_t* successor;  // [vocab, top]
  int64_t vocab;
  int top;
  const int64_t* stale;  // [B]
  int64_t* tokens;       // [B, T]
  int64_t* chains;       // [B]
  int64_t* phases;       // [B, T]
  int count, d0, d1, d2, d3, maxlen;
  unsigned* err;
};

// rank of index i: i + (suffix agreement length - 1) * size for an earlier occurrence of the
// newest token, else -1 (spec.py:38-49)
__device__ __forceinline__ long long match_rank(const int64_t* h, long long i, long long place, long long size,
                                                int maxlen, int64_t last) {
  if (!(i < place && h[i] == last)) return -1;
  long long length = 1;
  for (int back = 1; back < maxlen; ++back) {
    const long long want_at = place - back > 0 ? place - back : 0;
    if (i < back || place < back || h[i - back] != h[want_at]) break;
    ++length;
  }
  return i + (length - 1) * size;
}

__device__ __forceinline__ long long block_max(long long v, long long* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const long long other = __shfl_xor_sync(0xffffffffu, v, o);
    v = other > v ? other : v;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // scratch may still be read by the previous reduction
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  long long best = scratch[0];
  for (int w = 1; w < kThreads / 32; ++w) best = scratch[w] > best ? scratch[w] : best;
  return best;
}

__global__ void __launch_bounds__(kThreads) propose_kernel(const ProposeParams p) {
  __shared__ long long scratch[kThreads / 32];
  __shared__ int64_t siblings[kMaxLanes];
  __shared__ int sibling_count;
  __shared__ int64_t first_draft;
  __shared__ int bad;
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  const int T = p.count;
  const int64_t* h = p.history + static_cast<size_t>(row) * p.size;
  const long long place = p.position[row];
  const long long size = p.size;
  if (threadIdx.x == 0) bad = !(place >= 0 && place < size);
  __syncthreads();
  if (bad) {
    if (threadIdx.x == 0) raise_error(p.err, kErrBadShape);
    return;
  }
  const int64_t last = h[place];
  long long best = -1;
  for (long long i = threadIdx.x; i < size; i += kThreads) {
    const long long r = match_rank(h, i, place, size, p.maxlen, last);
    best = r > best ? r : best;
  }
  best = block_max(best, scratch);
  const bool found = best >= 0;
  const long long start = found ? best % size : place;
  const long long matched = found ? best / size + 1 : 0;
  const int drafts = matched <= 1 ? p.d0 : matched <= 3 ? p.d1 : matched <= 7 ? p.d2 : p.d3;
  int64_t* out = p.tokens + static_cast<size_t>(row) * T;
  const int lanes = T - 1 - min(min(p.d0, p.d1), min(p.d2, p.d3));
  auto successor = [&](int64_t token, int entry) -> int64_t {
    if (token < 0 || token >= p.vocab) {
      raise_error(p.err, kErrBadShape);
      return 0;
    }
    return p.successor[token * p.top + entry];
  };
  if (threadIdx.x == 0) {
    out[0] = last;
    int64_t previous = last, first = last;
    for (int step = 1; step < T; ++step) {
      const long long source = start + step;
      const int64_t draft = (found && source <= place) ? h[source < size - 1 ? source : size - 1]
                                                       : successor(previous, 0);
      if (step <= drafts) out[step] = draft;
      previous = draft;
      if (step == 1) first = draft;
    }
    first_draft = first;
    int count = 0;
    const int64_t hint = p.stale[row];
    if (lanes > 0 && hint >= 0 && hint != first && T - 1 - drafts >= 2) siblings[count++] = hint;
    sibling_count = count;
  }
  __syncthreads();
  if (lanes > 0) {
    const int64_t first = first_draft;
    // Alternatives from other occurrences of the newest token: what followed the best-ranked
    // occurrence whose follower is neither draft 1 nor already a sibling, up to three times.
    const int rounds = lanes < 3 ? lanes : 3;
    for (int round = 0; round < rounds; ++round) {
      const int count = sibling_count;
      long long choice = -1;
      for (long long i = threadIdx.x; i < size; i += kThreads) {
        const long long r = match_rank(h, i, place, size, p.maxlen, last);
        if (r < 0) continue;
        const int64_t after = h[i + 1];  // i < place < size
        bool taken = after == first;
        for (int s = 0; s < count; ++s) taken = taken || siblings[s] == after;
        if (!taken) choice = r > choice ? r : choice;
      }
      choice = block_max(choice, scratch);
      if (threadIdx.x == 0 && choice >= 0 && count < lanes) {
        siblings[count] = h[choice % size + 1];
        sibling_count = count + 1;
      }
      __syncthreads();
    }
    if (threadIdx.x == 0) {
      int count = sibling_count;
      for (int entry = 0; entry < p.top; ++entry) {
        const int64_t candidate = successor(last, entry);
        bool fresh = candidate != first;
        for (int s = 0; s < count; ++s) fresh = fresh && siblings[s] != candidate;
        if (fresh && count < lanes) siblings[count++] = candidate;
      }
      for (int lane = 0; lane < lanes; ++lane)
        if (1 + drafts + lane < T) out[1 + drafts + lane] = lane < count ? siblings[lane] : first;
    }
  }
  if (threadIdx.x == 0) p.chains[row] = 1 + drafts;
  for (int slot = threadIdx.x; slot < T; slot += kThreads)
    p.phases[static_cast<size_t>(row) * T + slot] = slot <= drafts ? slot : 1;
}

__global__ void within_margin_kernel(const __nv_bfloat16* logits, int64_t vocab, const int64_t* tokens,
                                     const float* top, int64_t* within, int batch, int count, float margin,
                                     unsigned* err) {
  pdl_wait();
  pdl_trigger();
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(batch) * count) return;
  const int slot = static_cast<int>(idx % count);
  if (slot == 0) {
    within[idx] = 0;  // slot 0 is the trusted token, not a draft
    return;
  }
  const int64_t draft = tokens[idx];
  const int64_t previous = idx - 1;
  if (draft < 0 || draft >= vocab) {
    raise_error(err, kErrBadShape);
    within[idx] = 0;
    return;
  }
  const float value = __bfloat162float(logits[previous * vocab + draft]);
  within[idx] = value >= top[previous] - margin ? 1 : 0;
}

struct SettleParams {
  const int64_t* tokens;  // [B, T]
  const int64_t* greedy;  // [B, T]
  const int64_t* within;  // [B, T] or null (exact acceptance)
  int64_t* position;      // [B]
  const int64_t* limit;   // [B]
  int64_t* history;       // [B, size]
  int64_t size;
  int64_t* result;        // [B, T + 1]
  int64_t* move_from;     // [B]
  int64_t* move_to;       // [B]
  const int64_t* chains;  // [B]
  int64_t* stale;         // [B]
  int batch, count;
  unsigned* err;
};

__global__ void settle_kernel(const SettleParams p) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= p.batch) return;
  const int T = p.count;
  const int64_t* draft = p.tokens + static_cast<size_t>(row) * T;
  const int64_t* chosen = p.greedy + static_cast<size_t>(row) * T;
  const long long place = p.position[row];
  long long chain = p.chains[row];
  if (place < 0 || place + 1 + T > p.size || chain < 1 || chain > T) {
    raise_error(p.err, kErrBadShape);
    return;
  }
  // the first illegal chain draft ends the run; gained = kept + 1
  long long gained = chain;
  for (int slot = 1; slot < chain; ++slot) {
    const bool legal = p.within != nullptr ? p.within[static_cast<size_t>(row) * T + slot] != 0
                                           : draft[slot] == chosen[slot - 1];
    if (!legal) {
      gained = slot;
      break;
    }
  }
  const long long accepted = gained;
  long long hit = T;
  for (int slot = static_cast<int>(chain); slot < T; ++slot)
    if (draft[slot] == chosen[0]) {
      hit = slot;
      break;
    }
  long long room = p.limit[row] - place;
  if (room < 0) room = 0;
  const bool branch = gained == 1 && hit < T && room >= 2;
  const long long guess_at = gained < T - 1 ? gained : T - 1;
  p.stale[row] = (gained < chain && !branch) ? chosen[guess_at] : -1;
  gained = branch ? 2 : gained;
  if (gained > room) gained = room;
  const int64_t bonus = chosen[hit < T - 1 ? hit : T - 1];
  int64_t* out = p.result + static_cast<size_t>(row) * (T + 1);
  int64_t* hist = p.history + static_cast<size_t>(row) * p.size + place + 1;
  out[0] = gained;
  for (int slot = 0; slot < T; ++slot) {
    int64_t emitted = slot + 1 < accepted ? draft[slot + 1] : chosen[slot];
    if (branch && slot == 1) emitted = bonus;
    out[1 + slot] = emitted;
    hist[slot] = emitted;
  }
  p.move_from[row] = branch ? place + hit : -1;
  p.move_to[row] = place + 1;
  p.position[row] = place + gained;
}

// store [planes, B, Hkv, C, D] bf16 (planes = 2 x layers): one CTA per (plane, row), 16-byte
// copies of the row's slot move_from -> move_to for every head.
__global__ void relocate_kernel(__nv_bfloat16* store, int batch, int kv_heads, int capacity, int dim,
                                const int64_t* move_from, const int64_t* move_to, unsigned* err) {
  pdl_wait();
  pdl_trigger();
  const int plane = blockIdx.x, row = blockIdx.y;
  const long long source = move_from[row], target = move_to[row];
  if (source < 0) return;
  if (source >= capacity || target < 0 || target >= capacity) {
    if (threadIdx.x == 0 && plane == 0) raise_error(err, kErrBadShape);
    return;
  }
  const int chunks = dim / 8;
  for (int e = threadIdx.x; e < kv_heads * chunks; e += blockDim.x) {
    const int head = e / chunks, c = e % chunks;
    __nv_bfloat16* base = store + ((static_cast<size_t>(plane) * batch + row) * kv_heads + head) * capacity * dim;
    *reinterpret_cast<uint4*>(base + target * dim + c * 8) = *reinterpret_cast<const uint4*>(base + source * dim + c * 8);
  }
}

}  // namespace spec
}  // namespace fb

using namespace fb;

extern "C" int fb_spec_propose(const int64_t* history, int64_t size, const int64_t* position, const int64_t* successor,
                               int64_t vocab, int top, const int64_t* stale, int64_t* tokens, int64_t* chains,
                               int64_t* phases, int batch, int tokens_per_row, int d0, int d1, int d2, int d3,
                               int maxlen, void* stream) {
  if (!history || !position || !successor || !stale || !tokens || !chains || !phases) return FB_ERR_ARG;
  if (batch <= 0 || size <= 1 || vocab <= 0 || top <= 0 || maxlen <= 0) return FB_ERR_ARG;
  if (tokens_per_row < 1 || tokens_per_row > spec::kMaxTokens) return FB_ERR_SHAPE;
  for (int d : {d0, d1, d2, d3})
    if (d < 1 || d > tokens_per_row - 1) return FB_ERR_ARG;
  if (size > (1ll << 40)) return FB_ERR_SHAPE;
  spec::ProposeParams p{history, size, position, successor, vocab, top, stale, tokens, chains, phases,
                        tokens_per_row, d0, d1, d2, d3, maxlen, error_word()};
  return launch_ex(spec::propose_kernel, dim3(batch), dim3(spec::kThreads), 0, static_cast<cudaStream_t>(stream), 1,
                   p);
}

extern "C" int fb_spec_within_margin(const void* logits, int64_t vocab, const int64_t* tokens, const float* top,
                                     int64_t* within, int batch, int count, float margin, void* stream) {
  if (!logits || !tokens || !top || !within || batch <= 0 || count <= 0 || vocab <= 0) return FB_ERR_ARG;
  const int64_t n = static_cast<int64_t>(batch) * count;
  const int threads = 128;
  return launch_ex(spec::within_margin_kernel, dim3(static_cast<unsigned>((n + threads - 1) / threads)),
                   dim3(threads), 0, static_cast<cudaStream_t>(stream), 1,
                   static_cast<const __nv_bfloat16*>(logits), vocab, tokens, top, within, batch, count, margin,
                   error_word());
}

extern "C" int fb_spec_settle(const int64_t* tokens, const int64_t* greedy, const int64_t* within, int64_t* position,
                              const int64_t* limit, int64_t* history, int64_t size, int64_t* result,
                              int64_t* move_from, int64_t* move_to, const int64_t* chains, int64_t* stale, int batch,
                              int count, void* stream) {
  if (!tokens || !greedy || !position || !limit || !history || !result || !move_from || !move_to || !chains ||
      !stale)
    return FB_ERR_ARG;
  if (batch <= 0 || count <= 0 || size <= 0) return FB_ERR_ARG;
  if (count > spec::kMaxTokens) return FB_ERR_SHAPE;
  spec::SettleParams p{tokens, greedy, within, position, limit, history, size, result, move_from, move_to,
                       chains, stale, batch, count, error_word()};
  const int threads = 64;
  return launch_ex(spec::settle_kernel, dim3((batch + threads - 1) / threads), dim3(threads), 0,
                   static_cast<cudaStream_t>(stream), 1, p);
}

extern "C" int fb_spec_relocate(void* store, int planes, int batch, int kv_heads, int capacity, int head_dim,
                                const int64_t* move_from, const int64_t* move_to, void* stream) {
  if (!store || !move_from || !move_to || planes <= 0 || batch <= 0 || kv_heads <= 0 || capacity <= 0)
    return FB_ERR_ARG;
  if (head_dim <= 0 || head_dim % 8 != 0 || planes > 65535 || batch > 65535) return FB_ERR_SHAPE;
  return launch_ex(spec::relocate_kernel, dim3(planes, batch), dim3(128), 0, static_cast<cudaStream_t>(stream), 1,
                   static_cast<__nv_bfloat16*>(store), batch, kv_heads, capacity, head_dim, move_from, move_to,
                   error_word());
}

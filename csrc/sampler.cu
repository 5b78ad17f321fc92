// Fused temperature / top-k / top-p sampler with the sampled token's log-probability.
//
// One 1024-thread CTA per row of fp32 logits:
//  1. radix select (4 rounds of 8-bit histograms over order-preserving keys) finds
//     the k-th largest logit without sorting the 151,936-entry row;
//  2. the k survivors are gathered into shared memory and bitonic-sorted (desc);
//  3. softmax over the survivors at temperature T, inclusive prefix sum, nucleus
//     cut (cumulative <= top_p, the first entry always kept), renormalisation;
//  4. inverse-CDF draw with a Philox-4x32-10 uniform keyed by (seed, row, step),
//     so the draw is reproducible and independent of launch order.
// The step counter and the seed are read from device memory, so a captured CUDA
// graph can advance / reseed them between replays.  k <= 1024 (k = 0 or k > 1024 uses 1024).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "host_utils.h"
#include "peer.cuh"
#include "vlm_ops.h"

namespace vlm {

constexpr int kSampThreads = 1024;
constexpr int kEpiTopk = 7;  // gemm_sm100.cu EPI_TOPK
constexpr int kKMax = 1024;

VLM_DEV uint32_t ordered_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(kSampThreads) sample_kernel(const float* __restrict__ logits, int64_t ld, int V,
                                                              int64_t* __restrict__ tok_out, float* __restrict__ lp_out,
                                                              const int64_t* __restrict__ step_ptr, float inv_temp,
                                                              int k, float top_p, const int64_t* __restrict__ seed_ptr,
                                                              long long row_offset) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix;
  __shared__ int s_remaining, s_gt, s_eq;
  __shared__ float cv[kKMax];
  __shared__ int ci[kKMax];
  __shared__ float cum[kKMax];
  __shared__ int s_choice;
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x, tid = threadIdx.x;
  const float* x = logits + static_cast<int64_t>(row) * ld;
  k = min(k, V);

  // 1. radix select of the k-th largest key
  uint32_t prefix = 0, mask = 0;
  int remaining = k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += kSampThreads) hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < V; i += kSampThreads) {
      const uint32_t u = ordered_key(x[i]);
      if ((u & mask) == prefix) atomicAdd(&hist[(u >> shift) & 0xFFu], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      int c = 0;
      for (int bin = 255; bin >= 0; --bin) {
        const int h = static_cast<int>(hist[bin]);
        if (c + h >= remaining) {
          s_prefix = prefix | (static_cast<uint32_t>(bin) << shift);
          s_remaining = remaining - c;
          break;
        }
        c += h;
      }
      s_gt = 0;
      s_eq = 0;
    }
    __syncthreads();
    prefix = s_prefix;
    remaining = s_remaining;
    mask |= 0xFFu << shift;
  }
  const uint32_t kth = prefix;
  // 2. gather survivors: all keys > kth, then `remaining` keys == kth
  const int n_gt = k - remaining;
  for (int i = tid; i < V; i += kSampThreads) {
    const float f = x[i];
    const uint32_t u = ordered_key(f);
    if (u > kth) {
      const int slot = atomicAdd(&s_gt, 1);
      cv[slot] = f;
      ci[slot] = i;
    } else if (u == kth) {
      const int slot = atomicAdd(&s_eq, 1);
      if (slot < remaining) {
        cv[n_gt + slot] = f;
        ci[n_gt + slot] = i;
      }
    }
  }
  __syncthreads();
  int P = 1;
  while (P < k) P <<= 1;
  for (int i = k + tid; i < P; i += kSampThreads) {
    cv[i] = -INFINITY;
    ci[i] = 0x7fffffff;
  }
  __syncthreads();
  // bitonic sort, descending by value, ties by ascending index
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < P; i += kSampThreads) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const float a = cv[i], b = cv[j];
          const int ia = ci[i], ib = ci[j];
          const bool a_first = (a > b) || (a == b && ia < ib);
          if (desc != a_first) {
            cv[i] = b;
            cv[j] = a;
            ci[i] = ib;
            ci[j] = ia;
          }
        }
      }
      __syncthreads();
    }
  }
  // 3. tempered softmax over the survivors + inclusive prefix sum
  const float vmax = cv[0];
  for (int i = tid; i < kKMax; i += kSampThreads) cum[i] = i < k ? __expf((cv[i] - vmax) * inv_temp) : 0.f;
  __syncthreads();
  for (int off = 1; off < kKMax; off <<= 1) {
    float add = 0.f;
    if (tid >= off) add = cum[tid - off];
    __syncthreads();
    cum[tid] += add;
    __syncthreads();
  }
  const float total = cum[k - 1];
  // nucleus: kept set is a prefix (cum is monotone)
  __shared__ int s_keep;
  if (tid == 0) s_keep = k;
  __syncthreads();
  if (top_p > 0.f && top_p < 1.f) {
    if (tid == 0) s_keep = 1;
    __syncthreads();
    if (tid < k && cum[tid] / total <= top_p) atomicMax(&s_keep, tid + 1);
    __syncthreads();
  }
  const int keep = s_keep;
  const float kept_total = cum[keep - 1];
  // 4. inverse-CDF draw
  const unsigned int step = static_cast<unsigned int>(*step_ptr);
  const unsigned long long seed = static_cast<unsigned long long>(*seed_ptr);
  const float u = philox_uniform(seed, static_cast<unsigned long long>(row + row_offset), step) * kept_total;
  if (tid == 0) s_choice = keep - 1;
  __syncthreads();
  if (tid < keep) {
    const float prev = tid == 0 ? 0.f : cum[tid - 1];
    if (cum[tid] >= u && prev < u) atomicMin(&s_choice, tid);
  }
  __syncthreads();
  if (tid == 0) {
    const int c = s_choice;
    const float pc = (cum[c] - (c == 0 ? 0.f : cum[c - 1])) / kept_total;
    tok_out[row] = ci[c];
    lp_out[row] = logf(fmaxf(pc, 1e-30f));
  }
}

void sample(at::Tensor logits, at::Tensor tok, at::Tensor lp, at::Tensor step, at::Tensor seed, double temperature,
            int64_t top_k, double top_p, int64_t row_offset) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1, "sample: fp32 [B, V]");
  TORCH_CHECK(step.scalar_type() == at::kLong && step.is_cuda(), "sample: step must be an int64 CUDA tensor");
  TORCH_CHECK(seed.scalar_type() == at::kLong && seed.is_cuda(), "sample: seed must be an int64 CUDA tensor");
  TORCH_CHECK(temperature > 0, "sample: temperature must be positive");
  const int B = static_cast<int>(logits.size(0));
  if (B == 0) return;
  const c10::cuda::CUDAGuard g(logits.device());
  const int k = (top_k <= 0 || top_k > kKMax) ? kKMax : static_cast<int>(top_k);
  launch_pdl(sample_kernel, dim3(B), dim3(kSampThreads), 0, at::cuda::getCurrentCUDAStream(), logits.data_ptr<float>(),
             logits.stride(0), static_cast<int>(logits.size(1)), tok.data_ptr<int64_t>(), lp.data_ptr<float>(),
             step.data_ptr<int64_t>(), static_cast<float>(1.0 / temperature), k, static_cast<float>(top_p),
             seed.data_ptr<int64_t>(), static_cast<long long>(row_offset));
}

// ------------------------------------------------------------------ lm_head fused with the sampler
// The lm_head GEMM runs with the EPI_TOPK epilogue: per (row, 128-column tile) it keeps the k largest
// logits (value desc, index asc), so the fp32 [B, V] logits are never written.  One CTA per row then merges
// the tiles' candidates into the row's top k and finishes exactly as sample_kernel does for those k
// survivors: tempered softmax, inclusive prefix sum (the same Hillis-Steele order), nucleus cut, Philox
// draw, log-probability of the choice.  With the same GEMM tiling as the unfused lm_head the logits are
// bitwise the same, so both paths sample the same tokens.  Reference: core/sampling.py:198-204 and
// utils/vlm.py:227-258 (mask logits to top-k / top-p, then sample).
constexpr int kFusedTopkMax = 16;
constexpr int kMergeThreads = 256;

VLM_DEV bool cand_before(float a, int ia, float b, int ib) { return a > b || (a == b && ia < ib); }

// Vocab-parallel variant (tensor-parallel decode): each rank's lm_head GEMM covered its vocabulary shard,
// so its merge finds the shard's top k.  Every value travels with the decode step's tag in an 8-byte word
// (fp32 bits or the global token id in the low half, the tag in the high half); the rank stores its k
// survivors into its slot of every rank's buffer ([W][B][kFusedTopkMax] word pairs), polls its own buffer
// until all ranks' survivors carry the tag, and picks the row's global top k from the W x k of them.  The
// global top k of a row is the top k of the shards' top k, so every rank draws the token a single GPU
// would draw from the whole vocabulary.
struct TopkExchange {
  PeerTable slots;                       // per rank: this step's [W][B][kFusedTopkMax][2] u64 words
  const unsigned long long* epoch;       // device step counter (its low 32 bits are the tag)
  int voff, rank, world;
  int* err;
};

template <bool TP>
__global__ void __launch_bounds__(kMergeThreads) topk_merge_sample_kernel(
    const float* __restrict__ cand_v, const int* __restrict__ cand_i, int tiles, int k, int64_t* __restrict__ tok_out,
    float* __restrict__ lp_out, const int64_t* __restrict__ step_ptr, float inv_temp, float top_p,
    const int64_t* __restrict__ seed_ptr, long long row_offset, TopkExchange ex) {
  __shared__ float wv[kMergeThreads / 32];
  __shared__ int wi[kMergeThreads / 32];
  __shared__ int wt[kMergeThreads / 32];
  __shared__ float cv[kFusedTopkMax];
  __shared__ int ci[kFusedTopkMax];
  __shared__ int s_win;
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = tiles * k;
  const float* v = cand_v + static_cast<int64_t>(row) * n;
  const int* ix = cand_i + static_cast<int64_t>(row) * n;
  // 1. this thread's sorted top k of its strided share of the candidates
  float tv[kFusedTopkMax];
  int ti[kFusedTopkMax];
#pragma unroll
  for (int j = 0; j < kFusedTopkMax; ++j) {
    tv[j] = -INFINITY;
    ti[j] = 0x7fffffff;
  }
  float tvk = -INFINITY;  // tv[k - 1], ti[k - 1] in registers (every array index below is static)
  int tik = 0x7fffffff;
  for (int c = tid; c < n; c += kMergeThreads) {
    const float z = v[c];
    const int zi = ix[c];
    if (!cand_before(z, zi, tvk, tik)) continue;
    bool placed = false;
#pragma unroll
    for (int q = kFusedTopkMax - 1; q > 0; --q) {
      if (q < k && !placed) {
        if (cand_before(z, zi, tv[q - 1], ti[q - 1])) {
          tv[q] = tv[q - 1];
          ti[q] = ti[q - 1];
        } else {
          tv[q] = z;
          ti[q] = zi;
          placed = true;
        }
      }
    }
    if (!placed) {
      tv[0] = z;
      ti[0] = zi;
    }
#pragma unroll
    for (int q = 0; q < kFusedTopkMax; ++q)
      if (q == k - 1) {
        tvk = tv[q];
        tik = ti[q];
      }
  }
  // 2. k rounds of a block-wide arg-max over the threads' heads; the winner pops its head
  int head = 0;
  for (int r = 0; r < k; ++r) {
    float bv = head < k ? tv[0] : -INFINITY;
    int bi = head < k ? ti[0] : 0x7fffffff;
    int bt = tid;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      const int ot = __shfl_xor_sync(0xffffffffu, bt, off);
      if (cand_before(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
        bt = ot;
      }
    }
    if (lane == 0) {
      wv[warp] = bv;
      wi[warp] = bi;
      wt[warp] = bt;
    }
    __syncthreads();
    if (tid == 0) {
      float xv = wv[0];
      int xi = wi[0], xt = wt[0];
      for (int w = 1; w < kMergeThreads / 32; ++w)
        if (cand_before(wv[w], wi[w], xv, xi)) {
          xv = wv[w];
          xi = wi[w];
          xt = wt[w];
        }
      cv[r] = xv;
      ci[r] = xi;
      s_win = xt;
    }
    __syncthreads();
    if (tid == s_win) {  // pop the head (a shift of the sorted list)
#pragma unroll
      for (int j = 0; j < kFusedTopkMax - 1; ++j) {
        tv[j] = tv[j + 1];
        ti[j] = ti[j + 1];
      }
      tv[kFusedTopkMax - 1] = -INFINITY;
      ti[kFusedTopkMax - 1] = 0x7fffffff;
      ++head;
    }
    __syncthreads();
  }
  if constexpr (TP) {
    // 2b. publish this shard's survivors (global token ids) to every rank; gather every rank's
    __shared__ float gv[kMaxRanks * kFusedTopkMax];
    __shared__ int gi[kMaxRanks * kFusedTopkMax];
    __shared__ int s_ok;
    const unsigned long long tag = static_cast<unsigned long long>(static_cast<unsigned>(*ex.epoch)) << 32;
    const int B = static_cast<int>(gridDim.x);
    if (tid == 0) s_ok = 1;
    if (tid < k) {
      const unsigned long long w0 = tag | __float_as_uint(cv[tid]);
      const unsigned long long w1 = tag | static_cast<unsigned>(ci[tid] + ex.voff);
      const int64_t off = ((static_cast<int64_t>(ex.rank) * B + row) * kFusedTopkMax + tid) * 2;
      for (int p = 0; p < ex.world; ++p) {
        unsigned long long* dst = reinterpret_cast<unsigned long long*>(ex.slots.p[p]) + off;
        asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(dst), "l"(w0), "l"(w1) : "memory");
      }
    }
    __syncthreads();
    if (tid < ex.world * k) {
      const int p = tid / k, j = tid - p * k;
      const unsigned long long* src = reinterpret_cast<const unsigned long long*>(ex.slots.p[ex.rank]) +
                                      ((static_cast<int64_t>(p) * B + row) * kFusedTopkMax + j) * 2;
      unsigned long long w0, w1;
      const long long t0 = clock64();
      bool good = true;
      while (true) {
        asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(src) : "memory");
        if ((w0 >> 32) == (tag >> 32) && (w1 >> 32) == (tag >> 32)) break;
        if (clock64() - t0 > kPeerWait) {
          atomicCAS(ex.err, 0, kErrTimeoutPeer);
          good = false;
          break;
        }
      }
      gv[tid] = __uint_as_float(static_cast<unsigned>(w0));
      gi[tid] = static_cast<int>(static_cast<unsigned>(w1));
      if (!good) s_ok = 0;
    }
    __syncthreads();
    if (!s_ok) {
      if (tid == 0) {
        tok_out[row] = 0;
        lp_out[row] = 0.f;
      }
      return;
    }
    // 2c. the row's global top k: k selection passes over the W x k survivors (ids are unique)
    if (tid == 0) {
      float pv = INFINITY;
      int pi = -1;
      for (int r = 0; r < k; ++r) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int c = 0; c < ex.world * k; ++c)
          if (cand_before(pv, pi, gv[c], gi[c]) && cand_before(gv[c], gi[c], bv, bi)) {
            bv = gv[c];
            bi = gi[c];
          }
        cv[r] = bv;
        ci[r] = bi;
        pv = bv;
        pi = bi;
      }
    }
    __syncthreads();
  }
  // 3. tempered softmax over the survivors, inclusive prefix sum in sample_kernel's order, nucleus, draw
  if (tid == 0) {
    const float vmax = cv[0];
    float cum[kFusedTopkMax];
#pragma unroll
    for (int i = 0; i < kFusedTopkMax; ++i) cum[i] = i < k ? __expf((cv[i] - vmax) * inv_temp) : 0.f;
#pragma unroll
    for (int off = 1; off < kFusedTopkMax; off <<= 1) {
      float nxt[kFusedTopkMax];
#pragma unroll
      for (int i = 0; i < kFusedTopkMax; ++i) nxt[i] = cum[i] + (i >= off ? cum[i - off] : 0.f);
#pragma unroll
      for (int i = 0; i < kFusedTopkMax; ++i) cum[i] = nxt[i];
    }
    float total = 0.f;
#pragma unroll
    for (int i = 0; i < kFusedTopkMax; ++i)
      if (i == k - 1) total = cum[i];
    int keep = k;
    if (top_p > 0.f && top_p < 1.f) {
      keep = 1;
#pragma unroll
      for (int i = 0; i < kFusedTopkMax; ++i)
        if (i < k && cum[i] / total <= top_p) keep = max(keep, i + 1);
    }
    float kept_total = 0.f;
#pragma unroll
    for (int i = 0; i < kFusedTopkMax; ++i)
      if (i == keep - 1) kept_total = cum[i];
    const unsigned int step = static_cast<unsigned int>(*step_ptr);
    const unsigned long long seed = static_cast<unsigned long long>(*seed_ptr);
    const float u = philox_uniform(seed, static_cast<unsigned long long>(row + row_offset), step) * kept_total;
    int choice = keep - 1;
    float prev_c = 0.f, cur_c = 0.f;
#pragma unroll
    for (int i = kFusedTopkMax - 1; i >= 0; --i) {
      if (i < keep) {
        const float prev = i == 0 ? 0.f : cum[i - 1];
        if (cum[i] >= u && prev < u) choice = i;
      }
    }
#pragma unroll
    for (int i = 0; i < kFusedTopkMax; ++i)
      if (i == choice) {
        cur_c = cum[i];
        prev_c = i == 0 ? 0.f : cum[i - 1];
      }
    int tok = 0;
#pragma unroll
    for (int i = 0; i < kFusedTopkMax; ++i)
      if (i == choice) tok = ci[i];
    tok_out[row] = tok;
    lp_out[row] = logf(fmaxf((cur_c - prev_c) / kept_total, 1e-30f));
  }
}

void lm_head_sample(at::Tensor h, at::Tensor w, at::Tensor tok, at::Tensor lp, at::Tensor step, at::Tensor seed,
                    double temperature, int64_t top_k, double top_p, int64_t row_offset) {
  TORCH_CHECK(step.scalar_type() == at::kLong && step.is_cuda(), "lm_head_sample: step must be an int64 CUDA tensor");
  TORCH_CHECK(seed.scalar_type() == at::kLong && seed.is_cuda(), "lm_head_sample: seed must be an int64 CUDA tensor");
  TORCH_CHECK(temperature > 0, "lm_head_sample: temperature must be positive");
  TORCH_CHECK(top_k >= 1 && top_k <= kFusedTopkMax, "lm_head_sample: 1 <= top_k <= ", kFusedTopkMax);
  const int64_t B = h.size(0), V = w.size(0);
  if (B == 0) return;
  TORCH_CHECK(top_k <= V, "lm_head_sample: top_k larger than the vocabulary");
  const c10::cuda::CUDAGuard g(h.device());
  constexpr int kTile = 128;  // the unfused lm_head's tile width for decode-sized M: bitwise the same logits
  const int tiles = static_cast<int>((V + kTile - 1) / kTile);
  const int k = static_cast<int>(top_k);
  at::Tensor cv = at::empty({B, tiles, k}, h.options().dtype(at::kFloat));
  at::Tensor ci = at::empty({B, tiles, k}, h.options().dtype(at::kInt));
  VocabArgs va{nullptr, nullptr, nullptr, nullptr, nullptr, cv.data_ptr<float>()};
  va.cand_i = ci.data_ptr<int>();
  va.topk = k;
  gemm_ex(h, w, at::Tensor(), at::Tensor(), at::Tensor(), at::Tensor(), true, true, 1.0, kEpiTopk, false, &va, kTile,
          nullptr, nullptr);
  launch_pdl(topk_merge_sample_kernel<false>, dim3(static_cast<unsigned>(B)), dim3(kMergeThreads), 0,
             at::cuda::getCurrentCUDAStream(), cv.data_ptr<float>(), ci.data_ptr<int>(), tiles, k,
             tok.data_ptr<int64_t>(), lp.data_ptr<float>(), step.data_ptr<int64_t>(),
             static_cast<float>(1.0 / temperature), static_cast<float>(top_p), seed.data_ptr<int64_t>(),
             static_cast<long long>(row_offset), TopkExchange{});
}

void lm_head_sample_tp(at::Tensor h, at::Tensor w, int64_t vocab_offset, at::Tensor tok, at::Tensor lp,
                       at::Tensor step, at::Tensor seed, double temperature, int64_t top_k, double top_p,
                       int64_t row_offset, std::vector<int64_t> slots, int64_t slot_off_bytes, int64_t epoch_ptr,
                       int64_t rank) {
  TORCH_CHECK(step.scalar_type() == at::kLong && step.is_cuda(), "lm_head_sample_tp: step must be an int64 CUDA tensor");
  TORCH_CHECK(seed.scalar_type() == at::kLong && seed.is_cuda(), "lm_head_sample_tp: seed must be an int64 CUDA tensor");
  TORCH_CHECK(temperature > 0, "lm_head_sample_tp: temperature must be positive");
  TORCH_CHECK(top_k >= 1 && top_k <= kFusedTopkMax, "lm_head_sample_tp: 1 <= top_k <= ", kFusedTopkMax);
  const int64_t B = h.size(0), V = w.size(0);
  const int W = static_cast<int>(slots.size());
  if (B == 0) return;
  TORCH_CHECK(top_k <= V, "lm_head_sample_tp: top_k larger than the vocabulary shard");
  TORCH_CHECK(rank >= 0 && rank < W && slot_off_bytes % 16 == 0, "lm_head_sample_tp: rank / slot alignment");
  const c10::cuda::CUDAGuard g(h.device());
  constexpr int kTile = 128;
  const int tiles = static_cast<int>((V + kTile - 1) / kTile);
  const int k = static_cast<int>(top_k);
  at::Tensor cv = at::empty({B, tiles, k}, h.options().dtype(at::kFloat));
  at::Tensor ci = at::empty({B, tiles, k}, h.options().dtype(at::kInt));
  VocabArgs va{nullptr, nullptr, nullptr, nullptr, nullptr, cv.data_ptr<float>()};
  va.cand_i = ci.data_ptr<int>();
  va.topk = k;
  gemm_ex(h, w, at::Tensor(), at::Tensor(), at::Tensor(), at::Tensor(), true, true, 1.0, kEpiTopk, false, &va, kTile,
          nullptr, nullptr);
  TopkExchange ex{make_peer_table(slots, slot_off_bytes), reinterpret_cast<const unsigned long long*>(epoch_ptr),
                  static_cast<int>(vocab_offset), static_cast<int>(rank), W, err_word(h.device().index())};
  launch_pdl(topk_merge_sample_kernel<true>, dim3(static_cast<unsigned>(B)), dim3(kMergeThreads), 0,
             at::cuda::getCurrentCUDAStream(), cv.data_ptr<float>(), ci.data_ptr<int>(), tiles, k,
             tok.data_ptr<int64_t>(), lp.data_ptr<float>(), step.data_ptr<int64_t>(),
             static_cast<float>(1.0 / temperature), static_cast<float>(top_p), seed.data_ptr<int64_t>(),
             static_cast<long long>(row_offset), ex);
}

}  // namespace vlm

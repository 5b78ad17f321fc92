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
#include "vlm_ops.h"

namespace vlm {

constexpr int kSampThreads = 1024;
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

}  // namespace vlm

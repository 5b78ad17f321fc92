// Fused lm_head -> log-softmax -> token log-prob / entropy (forward and backward)
// over a 151,936-entry vocabulary without materialising fp32 logits.
//
// Forward: the tcgen05 GEMM runs with the VOCAB_STATS epilogue: each epilogue
// thread owns one row of a 128 x 256 logits tile in TMEM and reduces it to
// (max, sum exp, sum exp*z, target logit); a combine kernel merges the ~600
// per-tile partials of a row into lse, entropy = lse - E_p[z] and logp[target].
// Backward: rows are processed in chunks; the GEMM's VOCAB_GRAD epilogue writes
// dlogits = g_lp*(onehot - p) - g_ent*p*(log p + H) as bf16, then two GEMMs give
// dh = dlogits . W and dW += dlogits^T . h (fp32 accumulation).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "host_utils.h"
#include "vlm_ops.h"

namespace vlm {

constexpr int kVocabBN = 256;
constexpr int kEpiVocabStats = 4;
constexpr int kEpiVocabGrad = 5;

__global__ void vocab_combine_kernel(const float4* __restrict__ part, int tiles, int M, float* __restrict__ logp,
                                     float* __restrict__ ent, float* __restrict__ lse) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const float4* p = part + static_cast<int64_t>(row) * tiles;
  float mx = -INFINITY;
  for (int t = lane; t < tiles; t += 32) mx = fmaxf(mx, p[t].x);
  mx = warp_max(mx);
  float s = 0.f, sz = 0.f, zt = 0.f;
  int found = 0;
  for (int t = lane; t < tiles; t += 32) {
    const float4 v = p[t];
    const float sc = v.x == -INFINITY ? 0.f : __expf(v.x - mx);
    s += v.y * sc;
    sz += v.z * sc;
    if (!isnan(v.w)) {
      zt = v.w;
      found = 1;
    }
  }
  s = warp_sum(s);
  sz = warp_sum(sz);
  zt = warp_sum(found ? zt : 0.f);
  if (lane == 0) {
    const float l = mx + logf(s);
    lse[row] = l;
    ent[row] = l - sz / s;
    logp[row] = zt - l;
  }
}

void vocab_logprob_fwd(at::Tensor h, at::Tensor w, at::Tensor targets, at::Tensor logp, at::Tensor ent, at::Tensor lse) {
  TORCH_CHECK(targets.scalar_type() == at::kLong && targets.is_contiguous(), "vocab: int64 targets");
  const int64_t M = h.size(0), V = w.size(0);
  if (M == 0) return;
  const c10::cuda::CUDAGuard g(h.device());
  const int tiles = static_cast<int>((V + kVocabBN - 1) / kVocabBN);
  at::Tensor part = at::empty({M, tiles, 4}, h.options().dtype(at::kFloat));
  VocabArgs va{targets.data_ptr<int64_t>(), nullptr, nullptr, nullptr, nullptr, part.data_ptr<float>()};
  gemm_ex(h, w, at::Tensor(), at::Tensor(), at::Tensor(), at::Tensor(), true, true, 1.0, kEpiVocabStats, false, &va,
          kVocabBN, nullptr, nullptr);
  vocab_combine_kernel<<<static_cast<int>((M * 32 + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const float4*>(part.data_ptr<float>()), tiles, static_cast<int>(M), logp.data_ptr<float>(),
      ent.data_ptr<float>(), lse.data_ptr<float>());
  VLM_LAUNCHED();
}

void vocab_logprob_bwd(at::Tensor h, at::Tensor w, at::Tensor targets, at::Tensor lse, at::Tensor ent, at::Tensor g_lp,
                       at::Tensor g_ent, at::Tensor dh, at::Tensor dw) {
  TORCH_CHECK(dw.scalar_type() == at::kFloat && dw.is_contiguous(), "vocab bwd: fp32 weight grad accumulator");
  TORCH_CHECK(g_lp.is_contiguous() && g_ent.is_contiguous() && lse.is_contiguous() && ent.is_contiguous(),
              "vocab bwd: contiguous row data");
  const int64_t M = h.size(0), V = w.size(0);
  if (M == 0) return;
  const c10::cuda::CUDAGuard g(h.device());
  const int64_t chunk = std::min<int64_t>(M, 4096);
  at::Tensor dz = at::empty({chunk, V}, h.options());
  for (int64_t r0 = 0; r0 < M; r0 += chunk) {
    const int64_t mc = std::min(chunk, M - r0);
    at::Tensor hc = h.narrow(0, r0, mc);
    at::Tensor dzc = dz.narrow(0, 0, mc);
    VocabArgs va{targets.data_ptr<int64_t>() + r0, lse.data_ptr<float>() + r0, ent.data_ptr<float>() + r0,
                 g_lp.data_ptr<float>() + r0, g_ent.data_ptr<float>() + r0, nullptr};
    gemm_ex(hc, w, dzc, at::Tensor(), at::Tensor(), at::Tensor(), true, true, 1.0, kEpiVocabGrad, false, &va, kVocabBN,
            nullptr, nullptr);
    gemm(dzc, w, dh.narrow(0, r0, mc), at::Tensor(), at::Tensor(), at::Tensor(), true, false, 1.0, 0, false);
    gemm(dzc, hc, dw, at::Tensor(), at::Tensor(), at::Tensor(), false, false, 1.0, 0, true);
  }
}

}  // namespace vlm

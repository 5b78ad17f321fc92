// Memory-bound kernels: RMSNorm / LayerNorm, q/k-norm + MRoPE, ViT 2-D rotary,
// SwiGLU backward, embedding gather / scatter / backward, KV-cache writes, AdamW,
// sum of squares and the uint8 image patchifier.
//
// All kernels are one-pass-per-row (warp or block per row) with 16-byte vector
// accesses where the row is 8-element aligned, fp32 math and a single rounding
// to bf16 on the way out.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "kv_layout.cuh"
#include "host_utils.h"

namespace vlm {

using bf16 = __nv_bfloat16;

static inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream(); }
static inline int blocks_for(int64_t n, int per) { return static_cast<int>(std::min<int64_t>((n + per - 1) / per, 1 << 20)); }

// ------------------------------------------------------------------ RMSNorm
// y = w * bf16(x * rstd): the normalised row is rounded to the input dtype before the
// weight multiply, as the HF Qwen3 RMSNorm does.
__global__ void rms_norm_fwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w, bf16* __restrict__ y,
                                    float* __restrict__ rstd, int M, int H, float eps) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
    const bf16* xr = x + static_cast<int64_t>(row) * H;
    float ss = 0.f;
    for (int c = lane * 8; c < H; c += 256) {
      const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(u[j]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / H + eps);
    if (lane == 0 && rstd) rstd[row] = r;
    bf16* yr = y + static_cast<int64_t>(row) * H;
    for (int c = lane * 8; c < H; c += 256) {
      const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
      const uint4 wv = *reinterpret_cast<const uint4*>(w + c);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w}, uw[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(u[j]), g = unpack_bf16x2(uw[j]);
        o[j] = pack_bf16x2(bf2f(f2bf(f.x * r)) * g.x, bf2f(f2bf(f.y * r)) * g.y);
      }
      *reinterpret_cast<uint4*>(yr + c) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// dx = r * (g - xhat * mean(g * xhat)),  g = dy * w;  dw += sum_rows dy * xhat
// One warp per row (grid-stride).  The weight gradient sum_rows(dy * xhat) accumulates in one [H] slice of
// shared memory per block through shared-memory atomics, which the block adds to dw once at the end (a
// per-block partial buffer summed by a second kernel measured slower: 57 vs 47 us at 5112 x 2560).  The
// slice is stored transposed, column c at (c % 8) * (H / 8) + c / 8: lane l owns columns 8l .. 8l+7 of each
// 256-column step, so the 32 lanes' updates of one element index fall in 32 consecutive words (no bank
// conflicts).  A 10 KB slice (H = 2560) leaves room for several blocks per SM, and the column loops are
// unrolled so that each warp keeps several rows' worth of 16-byte loads in flight.
// ``add`` (optional) is a second gradient for the same tensor (the residual path), summed before rounding.
__global__ void rms_norm_bwd_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ x, const bf16* __restrict__ w,
                                    const float* __restrict__ rstd, const bf16* __restrict__ add,
                                    bf16* __restrict__ dx, float* __restrict__ dw, int M, int H) {
  extern __shared__ float sdw[];  // [H] when dw
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int H8 = H >> 3;
  if (dw)
    for (int c = threadIdx.x; c < H; c += blockDim.x) sdw[c] = 0.f;
  __syncthreads();
  for (int row = blockIdx.x * warps + wid; row < M; row += gridDim.x * warps) {
    const bf16* xr = x + static_cast<int64_t>(row) * H;
    const bf16* dyr = dy + static_cast<int64_t>(row) * H;
    const float r = rstd[row];
    float dot = 0.f;
#pragma unroll 4
    for (int c = lane * 8; c < H; c += 256) {
      const uint4 a = *reinterpret_cast<const uint4*>(xr + c), b = *reinterpret_cast<const uint4*>(dyr + c),
                  ww = *reinterpret_cast<const uint4*>(w + c);
      const uint32_t ua[4] = {a.x, a.y, a.z, a.w}, ub[4] = {b.x, b.y, b.z, b.w}, uw[4] = {ww.x, ww.y, ww.z, ww.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 fx = unpack_bf16x2(ua[j]), fd = unpack_bf16x2(ub[j]), fw = unpack_bf16x2(uw[j]);
        dot += fd.x * fw.x * fx.x * r + fd.y * fw.y * fx.y * r;
        if (dw) {
          atomicAdd(&sdw[(2 * j) * H8 + (c >> 3)], fd.x * fx.x * r);
          atomicAdd(&sdw[(2 * j + 1) * H8 + (c >> 3)], fd.y * fx.y * r);
        }
      }
    }
    dot = warp_sum(dot) / H;
    bf16* dxr = dx + static_cast<int64_t>(row) * H;
    const bf16* ar = add ? add + static_cast<int64_t>(row) * H : nullptr;
#pragma unroll 4
    for (int c = lane * 8; c < H; c += 256) {
      const uint4 a = *reinterpret_cast<const uint4*>(xr + c), b = *reinterpret_cast<const uint4*>(dyr + c),
                  ww = *reinterpret_cast<const uint4*>(w + c);
      const uint32_t ua[4] = {a.x, a.y, a.z, a.w}, ub[4] = {b.x, b.y, b.z, b.w}, uw[4] = {ww.x, ww.y, ww.z, ww.w};
      uint32_t ue[4] = {0u, 0u, 0u, 0u};
      if (ar) {
        const uint4 e = *reinterpret_cast<const uint4*>(ar + c);
        ue[0] = e.x;
        ue[1] = e.y;
        ue[2] = e.z;
        ue[3] = e.w;
      }
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 fx = unpack_bf16x2(ua[j]), fd = unpack_bf16x2(ub[j]), fw = unpack_bf16x2(uw[j]);
        const float2 fe = unpack_bf16x2(ue[j]);
        o[j] = pack_bf16x2(r * (fd.x * fw.x - fx.x * r * dot) + fe.x, r * (fd.y * fw.y - fx.y * r * dot) + fe.y);
      }
      *reinterpret_cast<uint4*>(dxr + c) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  if (dw) {
    __syncthreads();
    for (int c = threadIdx.x; c < H; c += blockDim.x) atomicAdd(&dw[c], sdw[(c & 7) * H8 + (c >> 3)]);
  }
}

// Small-M variant (decode): one CTA per row, one 16-byte chunk per thread held in registers.
__global__ void rms_norm_row_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w, bf16* __restrict__ y,
                                    float* __restrict__ rstd, int H, float eps) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x, c = threadIdx.x * 8;
  __shared__ float red[32];
  const bf16* xr = x + static_cast<int64_t>(row) * H;
  uint4 v = make_uint4(0, 0, 0, 0);
  float ss = 0.f;
  if (c < H) {
    v = *reinterpret_cast<const uint4*>(xr + c);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(u[j]);
      ss += f.x * f.x + f.y * f.y;
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x + 31) / 32 ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float r = rsqrtf(red[0] / H + eps);
  if (threadIdx.x == 0 && rstd) rstd[row] = r;
  if (c < H) {
    const uint4 wv = *reinterpret_cast<const uint4*>(w + c);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w}, uw[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(u[j]), g = unpack_bf16x2(uw[j]);
      o[j] = pack_bf16x2(bf2f(f2bf(f.x * r)) * g.x, bf2f(f2bf(f.y * r)) * g.y);
    }
    *reinterpret_cast<uint4*>(y + static_cast<int64_t>(row) * H + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

void rms_norm_fwd(at::Tensor x, at::Tensor w, at::Tensor y, at::Tensor rstd, double eps) {
  TORCH_CHECK(x.is_contiguous() && x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "rms_norm: bf16");
  const int H = static_cast<int>(x.size(-1));
  const int M = static_cast<int>(x.numel() / H);
  TORCH_CHECK(H % 8 == 0, "rms_norm: hidden size must be a multiple of 8");
  if (M == 0) return;
  const c10::cuda::CUDAGuard g(x.device());
  if (M < 1024 && H <= 8192) {
    const int threads = ((H / 8 + 31) / 32) * 32;
    launch_pdl(rms_norm_row_kernel, dim3(M), dim3(threads), 0, cur_stream(), reinterpret_cast<const bf16*>(x.data_ptr()),
               reinterpret_cast<const bf16*>(w.data_ptr()), reinterpret_cast<bf16*>(y.data_ptr()),
               rstd.defined() && rstd.numel() ? rstd.data_ptr<float>() : nullptr, H, static_cast<float>(eps));
    return;
  }
  rms_norm_fwd_kernel<<<blocks_for(M, 8), 256, 0, cur_stream()>>>(
      reinterpret_cast<const bf16*>(x.data_ptr()), reinterpret_cast<const bf16*>(w.data_ptr()),
      reinterpret_cast<bf16*>(y.data_ptr()), rstd.defined() && rstd.numel() ? rstd.data_ptr<float>() : nullptr, M, H,
      static_cast<float>(eps));
  VLM_LAUNCHED();
}

void rms_norm_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd, at::Tensor dx, at::Tensor dw,
                  at::Tensor add) {
  const int H = static_cast<int>(x.size(-1));
  const int M = static_cast<int>(x.numel() / H);
  if (M == 0) return;
  TORCH_CHECK(dy.is_contiguous() && x.is_contiguous() && H % 8 == 0, "rms_norm_bwd: contiguous inputs, H % 8 == 0");
  const bool has_add = add.defined() && add.numel();
  TORCH_CHECK(!has_add || (add.is_contiguous() && add.numel() == x.numel() && add.scalar_type() == at::kBFloat16),
              "rms_norm_bwd: bad residual gradient");
  const c10::cuda::CUDAGuard g(x.device());
  const bool has_dw = dw.defined() && dw.numel();
  TORCH_CHECK(!has_dw || (dw.scalar_type() == at::kFloat && dw.is_contiguous() && dw.numel() == H),
              "rms_norm_bwd: dw must be a contiguous fp32 [H] accumulator");
  constexpr int kThreads = 256;
  const int smem = has_dw ? H * static_cast<int>(sizeof(float)) : 0;
  if (smem > 48 * 1024)
    VLM_CUDA_CHECK(cudaFuncSetAttribute(rms_norm_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int blocks = std::min(blocks_for(M, 8), num_sms(x.device().index()) * (smem > 56 * 1024 ? 1 : 4));
  rms_norm_bwd_kernel<<<blocks, kThreads, smem, cur_stream()>>>(
      reinterpret_cast<const bf16*>(dy.data_ptr()), reinterpret_cast<const bf16*>(x.data_ptr()),
      reinterpret_cast<const bf16*>(w.data_ptr()), rstd.data_ptr<float>(),
      has_add ? reinterpret_cast<const bf16*>(add.data_ptr()) : nullptr, reinterpret_cast<bf16*>(dx.data_ptr()),
      has_dw ? dw.data_ptr<float>() : nullptr, M, H);
  VLM_LAUNCHED();
}

// ------------------------------------------------------------------ LayerNorm (ViT, forward only)
__global__ void layer_norm_fwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w, const bf16* __restrict__ b,
                                      bf16* __restrict__ y, int M, int H, float eps) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
    const bf16* xr = x + static_cast<int64_t>(row) * H;
    float s = 0.f;
    for (int c = lane; c < H; c += 32) s += bf2f(xr[c]);
    const float mean = warp_sum(s) / H;
    float v = 0.f;
    for (int c = lane; c < H; c += 32) {
      const float d = bf2f(xr[c]) - mean;
      v += d * d;
    }
    const float r = rsqrtf(warp_sum(v) / H + eps);
    bf16* yr = y + static_cast<int64_t>(row) * H;
    for (int c = lane; c < H; c += 32) yr[c] = f2bf((bf2f(xr[c]) - mean) * r * bf2f(w[c]) + (b ? bf2f(b[c]) : 0.f));
  }
}

void layer_norm_fwd(at::Tensor x, at::Tensor w, at::Tensor b, at::Tensor y, double eps) {
  const int H = static_cast<int>(x.size(-1));
  const int M = static_cast<int>(x.numel() / H);
  if (M == 0) return;
  TORCH_CHECK(x.is_contiguous(), "layer_norm: contiguous input");
  const c10::cuda::CUDAGuard g(x.device());
  layer_norm_fwd_kernel<<<blocks_for(M, 8), 256, 0, cur_stream()>>>(
      reinterpret_cast<const bf16*>(x.data_ptr()), reinterpret_cast<const bf16*>(w.data_ptr()),
      b.defined() && b.numel() ? reinterpret_cast<const bf16*>(b.data_ptr()) : nullptr,
      reinterpret_cast<bf16*>(y.data_ptr()), M, H, static_cast<float>(eps));
  VLM_LAUNCHED();
}

// ------------------------------------------------------------------ q/k RMSNorm + MRoPE
// One warp per (token, head).  Heads [0, nq) are q, [nq, nq+nkv) are k, the rest v (copied).
// Frequency j of the rotate-half pair (j, j + D/2) uses position axis ax[j] and inv_freq[j].
__global__ void qk_norm_rope_fwd_kernel(const bf16* __restrict__ qkv, const bf16* __restrict__ qw,
                                        const bf16* __restrict__ kw, const int* __restrict__ pos, int64_t pos_stride,
                                        const float* __restrict__ inv_freq, const int* __restrict__ ax,
                                        bf16* __restrict__ q, bf16* __restrict__ k, bf16* __restrict__ v,
                                        float* __restrict__ rq, float* __restrict__ rk, int T, int nq, int nkv, int D,
                                        float eps) {
  const int nh = nq + 2 * nkv;
  const int lane = threadIdx.x & 31;
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (gw >= static_cast<int64_t>(T) * nh) return;
  const int t = static_cast<int>(gw / nh), h = static_cast<int>(gw % nh);
  const bf16* src = qkv + (static_cast<int64_t>(t) * nh + h) * D;
  if (h >= nq + nkv) {
    bf16* dst = v + (static_cast<int64_t>(t) * nkv + (h - nq - nkv)) * D;
    for (int c = lane; c < D; c += 32) dst[c] = src[c];
    return;
  }
  const bool is_q = h < nq;
  const bool norm = qw != nullptr;  // Qwen2.5-style attention has no q/k RMSNorm: rotate only
  float ss = 0.f;
  if (norm)
    for (int c = lane; c < D; c += 32) {
      const float f = bf2f(src[c]);
      ss += f * f;
    }
  const float r = norm ? rsqrtf(warp_sum(ss) / D + eps) : 1.f;
  const bf16* wt = is_q ? qw : kw;
  bf16* dst = is_q ? q + (static_cast<int64_t>(t) * nq + h) * D : k + (static_cast<int64_t>(t) * nkv + (h - nq)) * D;
  if (lane == 0) {
    if (is_q)
      rq[static_cast<int64_t>(t) * nq + h] = r;
    else
      rk[static_cast<int64_t>(t) * nkv + (h - nq)] = r;
  }
  const int half = D / 2;
  for (int j = lane; j < half; j += 32) {
    const float x1 = bf2f(src[j]) * r * (norm ? bf2f(wt[j]) : 1.f);
    const float x2 = bf2f(src[j + half]) * r * (norm ? bf2f(wt[j + half]) : 1.f);
    const float p = static_cast<float>(pos[ax[j] * pos_stride + t]);
    float s, c;
    sincosf(p * inv_freq[j], &s, &c);
    dst[j] = f2bf(x1 * c - x2 * s);
    dst[j + half] = f2bf(x2 * c + x1 * s);
  }
}

// The same forward for D = 64 and 128.  A warp takes HPW = 4 consecutive heads of one token; each lane holds
// PER = D/64 adjacent rotation pairs of every one of them.  All heads' elements are requested before any is
// used (bf16x2 words when PER = 2), and the angles, which depend on the token and the pair only, are
// computed once per warp for its four heads (the scalar kernel above reads 2-byte elements twice and
// evaluates sincos per head).
template <int D>
__global__ void __launch_bounds__(256) qk_norm_rope_fwd_vec_kernel(
    const bf16* __restrict__ qkv, const bf16* __restrict__ qw, const bf16* __restrict__ kw,
    const int* __restrict__ pos, int64_t pos_stride, const float* __restrict__ inv_freq, const int* __restrict__ ax,
    bf16* __restrict__ q, bf16* __restrict__ k, bf16* __restrict__ v, float* __restrict__ rq, float* __restrict__ rk,
    int T, int nq, int nkv, float eps) {
  constexpr int HALF = D / 2, PER = HALF / 32, HPW = 4;
  static_assert(PER == 1 || PER == 2, "D = 64 or 128");
  const int nh = nq + 2 * nkv;
  const int groups = (nh + HPW - 1) / HPW;
  const int lane = threadIdx.x & 31;
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (gw >= static_cast<int64_t>(T) * groups) return;
  const int t = static_cast<int>(gw / groups), h0 = static_cast<int>(gw % groups) * HPW;
  const int j0 = lane * PER;
  const bf16* row = qkv + static_cast<int64_t>(t) * nh * D;
  float x1[HPW][PER], x2[HPW][PER];
#pragma unroll
  for (int e = 0; e < HPW; ++e) {
    const int h = min(h0 + e, nh - 1);  // a ragged last group re-reads its last head and skips it below
    const bf16* src = row + static_cast<int64_t>(h) * D;
    if constexpr (PER == 2) {
      const float2 a = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(src + j0));
      const float2 b = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(src + HALF + j0));
      x1[e][0] = a.x;
      x1[e][1] = a.y;
      x2[e][0] = b.x;
      x2[e][1] = b.y;
    } else {
      x1[e][0] = bf2f(src[j0]);
      x2[e][0] = bf2f(src[HALF + j0]);
    }
  }
  float sn[PER], cs[PER];
  bool angles = false;
  const bool norm = qw != nullptr;  // Qwen2.5-style attention has no q/k RMSNorm: rotate only
#pragma unroll
  for (int e = 0; e < HPW; ++e) {
    const int h = h0 + e;
    if (h >= nh) break;
    if (h >= nq + nkv) {  // v: a plain copy
      bf16* dst = v + (static_cast<int64_t>(t) * nkv + (h - nq - nkv)) * D;
      if constexpr (PER == 2) {
        *reinterpret_cast<uint32_t*>(dst + j0) = pack_bf16x2(x1[e][0], x1[e][1]);
        *reinterpret_cast<uint32_t*>(dst + HALF + j0) = pack_bf16x2(x2[e][0], x2[e][1]);
      } else {
        dst[j0] = f2bf(x1[e][0]);
        dst[HALF + j0] = f2bf(x2[e][0]);
      }
      continue;
    }
    if (!angles) {
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int j = j0 + i;
        sincosf(static_cast<float>(pos[ax[j] * pos_stride + t]) * inv_freq[j], &sn[i], &cs[i]);
      }
      angles = true;
    }
    const bool is_q = h < nq;
    float r = 1.f;
    float a1[PER], a2[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      a1[i] = x1[e][i];
      a2[i] = x2[e][i];
    }
    if (norm) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < PER; ++i) ss += a1[i] * a1[i] + a2[i] * a2[i];
      r = rsqrtf(warp_sum(ss) / D + eps);
      const bf16* wt = is_q ? qw : kw;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        a1[i] *= r * bf2f(wt[j0 + i]);
        a2[i] *= r * bf2f(wt[HALF + j0 + i]);
      }
    }
    bf16* dst = is_q ? q + (static_cast<int64_t>(t) * nq + h) * D : k + (static_cast<int64_t>(t) * nkv + (h - nq)) * D;
    if (lane == 0) {
      if (is_q)
        rq[static_cast<int64_t>(t) * nq + h] = r;
      else
        rk[static_cast<int64_t>(t) * nkv + (h - nq)] = r;
    }
    float o1[PER], o2[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      o1[i] = a1[i] * cs[i] - a2[i] * sn[i];
      o2[i] = a2[i] * cs[i] + a1[i] * sn[i];
    }
    if constexpr (PER == 2) {
      *reinterpret_cast<uint32_t*>(dst + j0) = pack_bf16x2(o1[0], o1[1]);
      *reinterpret_cast<uint32_t*>(dst + HALF + j0) = pack_bf16x2(o2[0], o2[1]);
    } else {
      dst[j0] = f2bf(o1[0]);
      dst[HALF + j0] = f2bf(o2[0]);
    }
  }
}

// Backward: un-rotate the incoming gradient, then the per-head RMSNorm backward.
// One warp per (token, head) item, grid-stride over items.  Lane l owns elements l + 32 i of a head, so
// the norm-weight gradient (sum over tokens and heads of g * xhat) accumulates in registers across the
// warp's items and reaches shared memory once per warp and global memory once per block.
template <int D>
__global__ void __launch_bounds__(256) qk_norm_rope_bwd_kernel(
    const bf16* __restrict__ dq, const bf16* __restrict__ dk, const bf16* __restrict__ dv,
    const bf16* __restrict__ qkv, const bf16* __restrict__ qw, const bf16* __restrict__ kw,
    const int* __restrict__ pos, int64_t pos_stride, const float* __restrict__ inv_freq, const int* __restrict__ ax,
    const float* __restrict__ rq, const float* __restrict__ rk, bf16* __restrict__ dqkv, float* __restrict__ dqw,
    float* __restrict__ dkw, int T, int nq, int nkv) {
  constexpr int HALF = D / 2;
  constexpr int PER = (HALF + 31) / 32;  // pair slots per lane
  __shared__ float sw[2 * D];            // q then k norm-weight gradient partials of this block
  for (int i = threadIdx.x; i < 2 * D; i += blockDim.x) sw[i] = 0.f;
  __syncthreads();
  const int nh = nq + 2 * nkv;
  const int lane = threadIdx.x & 31;
  const bool norm = qw != nullptr;
  float accq[2 * PER], acck[2 * PER];
#pragma unroll
  for (int i = 0; i < 2 * PER; ++i) accq[i] = acck[i] = 0.f;
  const int64_t items = static_cast<int64_t>(T) * nh;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; gw < items; gw += nwarps) {
    const int t = static_cast<int>(gw / nh), h = static_cast<int>(gw % nh);
    bf16* out = dqkv + (static_cast<int64_t>(t) * nh + h) * D;
    if (h >= nq + nkv) {
      const bf16* g = dv + (static_cast<int64_t>(t) * nkv + (h - nq - nkv)) * D;
      for (int c = lane; c < D; c += 32) out[c] = g[c];
      continue;
    }
    const bool is_q = h < nq;
    const bf16* g = is_q ? dq + (static_cast<int64_t>(t) * nq + h) * D : dk + (static_cast<int64_t>(t) * nkv + h - nq) * D;
    const bf16* x = qkv + (static_cast<int64_t>(t) * nh + h) * D;
    float n1[PER], n2[PER], xh1[PER], xh2[PER];
    float dot = 0.f;
    const float r = norm ? (is_q ? rq[static_cast<int64_t>(t) * nq + h] : rk[static_cast<int64_t>(t) * nkv + h - nq]) : 1.f;
    const bf16* wt = is_q ? qw : kw;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int j = lane + 32 * i;
      n1[i] = n2[i] = xh1[i] = xh2[i] = 0.f;
      if (j < HALF) {
        const float p = static_cast<float>(pos[ax[j] * pos_stride + t]);
        float s, c;
        sincosf(p * inv_freq[j], &s, &c);
        const float g1 = bf2f(g[j]), g2 = bf2f(g[j + HALF]);
        n1[i] = g1 * c + g2 * s;  // rotate back by the same angle
        n2[i] = g2 * c - g1 * s;
        if (norm) {
          xh1[i] = bf2f(x[j]) * r;
          xh2[i] = bf2f(x[j + HALF]) * r;
          dot += n1[i] * bf2f(wt[j]) * xh1[i] + n2[i] * bf2f(wt[j + HALF]) * xh2[i];
        }
      }
    }
    if (!norm) {
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int j = lane + 32 * i;
        if (j < HALF) {
          out[j] = f2bf(n1[i]);
          out[j + HALF] = f2bf(n2[i]);
        }
      }
      continue;
    }
    dot = warp_sum(dot) / D;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int j = lane + 32 * i;
      if (j < HALF) {
        out[j] = f2bf(r * (n1[i] * bf2f(wt[j]) - xh1[i] * dot));
        out[j + HALF] = f2bf(r * (n2[i] * bf2f(wt[j + HALF]) - xh2[i] * dot));
        float* acc = is_q ? accq : acck;
        acc[2 * i] += n1[i] * xh1[i];
        acc[2 * i + 1] += n2[i] * xh2[i];
      }
    }
  }
  if (norm) {
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int j = lane + 32 * i;
      if (j < HALF) {
        atomicAdd(&sw[j], accq[2 * i]);
        atomicAdd(&sw[j + HALF], accq[2 * i + 1]);
        atomicAdd(&sw[D + j], acck[2 * i]);
        atomicAdd(&sw[D + j + HALF], acck[2 * i + 1]);
      }
    }
  }
  __syncthreads();
  if (norm)
    for (int i = threadIdx.x; i < 2 * D; i += blockDim.x) {
      float* dst = i < D ? dqw : dkw;
      if (dst) atomicAdd(&dst[i % D], sw[i]);
    }
}

// Undefined or empty weight tensors select the rotation-only variant (no q/k RMSNorm).
static const bf16* opt_bf16(const at::Tensor& t) {
  return t.defined() && t.numel() ? reinterpret_cast<const bf16*>(t.data_ptr()) : nullptr;
}

void qk_norm_rope_fwd(at::Tensor qkv, at::Tensor qw, at::Tensor kw, at::Tensor pos, at::Tensor inv_freq, at::Tensor ax,
                      at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor rq, at::Tensor rk, int64_t nq, int64_t nkv,
                      double eps) {
  const int T = static_cast<int>(qkv.size(0));
  const int D = static_cast<int>(q.size(-1));
  if (T == 0) return;
  TORCH_CHECK(qkv.is_contiguous() && pos.scalar_type() == at::kInt && pos.dim() == 2 && pos.stride(1) == 1,
              "qk_norm_rope: layout");
  const c10::cuda::CUDAGuard g(qkv.device());
  const int64_t warps = static_cast<int64_t>(T) * (nq + 2 * nkv);
  static const bool vec = [] {  // VLMRL_QK_ROPE_VEC=0 keeps the scalar kernel (for A/B timing)
    const char* e = std::getenv("VLMRL_QK_ROPE_VEC");
    return !(e && e[0] == '0');
  }();
  if (vec && (D == 64 || D == 128)) {
    auto kern = D == 128 ? qk_norm_rope_fwd_vec_kernel<128> : qk_norm_rope_fwd_vec_kernel<64>;
    const int64_t vwarps = static_cast<int64_t>(T) * ((nq + 2 * nkv + 3) / 4);
    kern<<<static_cast<int>((vwarps * 32 + 255) / 256), 256, 0, cur_stream()>>>(
        reinterpret_cast<const bf16*>(qkv.data_ptr()), opt_bf16(qw), opt_bf16(kw), pos.data_ptr<int>(), pos.stride(0),
        inv_freq.data_ptr<float>(), ax.data_ptr<int>(), reinterpret_cast<bf16*>(q.data_ptr()),
        reinterpret_cast<bf16*>(k.data_ptr()), reinterpret_cast<bf16*>(v.data_ptr()), rq.data_ptr<float>(),
        rk.data_ptr<float>(), T, static_cast<int>(nq), static_cast<int>(nkv), static_cast<float>(eps));
    VLM_LAUNCHED();
    return;
  }
  qk_norm_rope_fwd_kernel<<<static_cast<int>((warps * 32 + 255) / 256), 256, 0, cur_stream()>>>(
      reinterpret_cast<const bf16*>(qkv.data_ptr()), opt_bf16(qw), opt_bf16(kw), pos.data_ptr<int>(), pos.stride(0),
      inv_freq.data_ptr<float>(), ax.data_ptr<int>(), reinterpret_cast<bf16*>(q.data_ptr()), reinterpret_cast<bf16*>(k.data_ptr()),
      reinterpret_cast<bf16*>(v.data_ptr()), rq.data_ptr<float>(), rk.data_ptr<float>(), T, static_cast<int>(nq),
      static_cast<int>(nkv), D, static_cast<float>(eps));
  VLM_LAUNCHED();
}

void qk_norm_rope_bwd(at::Tensor dq, at::Tensor dk, at::Tensor dv, at::Tensor qkv, at::Tensor qw, at::Tensor kw,
                      at::Tensor pos, at::Tensor inv_freq, at::Tensor ax, at::Tensor rq, at::Tensor rk, at::Tensor dqkv,
                      at::Tensor dqw, at::Tensor dkw, int64_t nq, int64_t nkv, double eps) {
  const int T = static_cast<int>(qkv.size(0));
  const int D = static_cast<int>(dq.size(-1));
  if (T == 0) return;
  TORCH_CHECK(dq.is_contiguous() && dk.is_contiguous() && dv.is_contiguous(), "qk_norm_rope_bwd: contiguous grads");
  const c10::cuda::CUDAGuard g(qkv.device());
  const int64_t warps = static_cast<int64_t>(T) * (nq + 2 * nkv);
  // enough warps to fill the GPU a few times; each loops over items so weight partials stay in registers
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((warps + 7) / 8, num_sms(qkv.device().index()) * 8)));
  auto args = [&](auto kern) {
    kern<<<blocks, 256, 0, cur_stream()>>>(
        reinterpret_cast<const bf16*>(dq.data_ptr()), reinterpret_cast<const bf16*>(dk.data_ptr()),
        reinterpret_cast<const bf16*>(dv.data_ptr()), reinterpret_cast<const bf16*>(qkv.data_ptr()), opt_bf16(qw),
        opt_bf16(kw), pos.data_ptr<int>(), pos.stride(0), inv_freq.data_ptr<float>(), ax.data_ptr<int>(),
        rq.data_ptr<float>(), rk.data_ptr<float>(), reinterpret_cast<bf16*>(dqkv.data_ptr()),
        dqw.defined() && dqw.numel() ? dqw.data_ptr<float>() : nullptr,
        dkw.defined() && dkw.numel() ? dkw.data_ptr<float>() : nullptr, T, static_cast<int>(nq), static_cast<int>(nkv));
  };
  switch (D) {
    case 32: args(qk_norm_rope_bwd_kernel<32>); break;
    case 64: args(qk_norm_rope_bwd_kernel<64>); break;
    case 80: args(qk_norm_rope_bwd_kernel<80>); break;
    case 128: args(qk_norm_rope_bwd_kernel<128>); break;
    case 256: args(qk_norm_rope_bwd_kernel<256>); break;
    default: TORCH_CHECK(false, "qk_norm_rope_bwd: unsupported head_dim ", D);
  }
  VLM_LAUNCHED();
}

// ------------------------------------------------------------------ ViT 2-D rotary
// qkv [N, 3, H, D] -> q, k (rotated), v.  Rotation pairs are (j, j+D/2).
//   style 0 (HF Qwen3-VL / Qwen2.5-VL): one angle per pair, (j < D/4 ? row : col) * 1e4^(-(j mod D/4)/(D/4)).
//   style 1 (the reference's Qwen3-VL tower, models/qwen3vl/vision.py:21-30,69-77): D/2 frequencies
//     1e4^(-j/(D/2)); element j uses row * f_j and element j+D/2 uses col * f_j (two angles per pair).
__global__ void vision_rope_kernel(const bf16* __restrict__ qkv, const int* __restrict__ rc, bf16* __restrict__ q,
                                   bf16* __restrict__ k, bf16* __restrict__ v, int N, int H, int D, int style) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int half = D / 2, quarter = D / 4;
  const int64_t total = static_cast<int64_t>(N) * H * half;
  if (idx >= total) return;
  const int j = static_cast<int>(idx % half);
  const int h = static_cast<int>((idx / half) % H);
  const int n = static_cast<int>(idx / (static_cast<int64_t>(half) * H));
  const int64_t base = static_cast<int64_t>(n) * 3 * H * D;
  const int64_t o = (static_cast<int64_t>(n) * H + h) * D;
  constexpr float kLog2Theta = 13.287712379549449f;  // log2(1e4)
  float s1, c1, s2, c2;
  if (style == 0) {
    const int coord = j < quarter ? rc[2 * n] : rc[2 * n + 1];
    const float freq = exp2f(-static_cast<float>(j % quarter) / quarter * kLog2Theta);
    sincosf(static_cast<float>(coord) * freq, &s1, &c1);
    s2 = s1;
    c2 = c1;
  } else {
    const float freq = exp2f(-static_cast<float>(j) / half * kLog2Theta);
    sincosf(static_cast<float>(rc[2 * n]) * freq, &s1, &c1);
    sincosf(static_cast<float>(rc[2 * n + 1]) * freq, &s2, &c2);
  }
#pragma unroll
  for (int which = 0; which < 2; ++which) {
    const bf16* src = qkv + base + static_cast<int64_t>(which) * H * D + static_cast<int64_t>(h) * D;
    bf16* dst = (which == 0 ? q : k) + o;
    const float x1 = bf2f(src[j]), x2 = bf2f(src[j + half]);
    dst[j] = f2bf(x1 * c1 - x2 * s1);
    dst[j + half] = f2bf(x2 * c2 + x1 * s2);
  }
  const bf16* sv = qkv + base + 2ll * H * D + static_cast<int64_t>(h) * D;
  v[o + j] = sv[j];
  v[o + j + half] = sv[j + half];
}

void vision_rope(at::Tensor qkv, at::Tensor rc, at::Tensor q, at::Tensor k, at::Tensor v, int64_t n_heads, int64_t style) {
  const int N = static_cast<int>(qkv.size(0));
  const int D = static_cast<int>(q.size(-1));
  if (N == 0) return;
  TORCH_CHECK(rc.scalar_type() == at::kInt && rc.is_contiguous(), "vision_rope: rc int32 [N,2]");
  TORCH_CHECK(style == 0 || style == 1, "vision_rope: style 0 (HF) or 1 (reference tower)");
  const c10::cuda::CUDAGuard g(qkv.device());
  const int64_t total = static_cast<int64_t>(N) * n_heads * (D / 2);
  vision_rope_kernel<<<static_cast<int>((total + 255) / 256), 256, 0, cur_stream()>>>(
      reinterpret_cast<const bf16*>(qkv.data_ptr()), rc.data_ptr<int>(), reinterpret_cast<bf16*>(q.data_ptr()),
      reinterpret_cast<bf16*>(k.data_ptr()), reinterpret_cast<bf16*>(v.data_ptr()), N, static_cast<int>(n_heads), D,
      static_cast<int>(style));
  VLM_LAUNCHED();
}

// ------------------------------------------------------------------ SwiGLU backward
// pre [M, 2F] interleaved (gate, up); d_act [M, F] -> d_pre [M, 2F]
__global__ void swiglu_bwd_kernel(const bf16* __restrict__ da, const bf16* __restrict__ pre, bf16* __restrict__ dpre,
                                  int64_t n_pairs) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n_pairs) return;
  const float2 gu = unpack_bf16x2(reinterpret_cast<const uint32_t*>(pre)[i]);
  const float g = gu.x, u = gu.y;
  const float s = 1.f / (1.f + __expf(-g));
  const float d = bf2f(da[i]);
  reinterpret_cast<uint32_t*>(dpre)[i] = pack_bf16x2(d * u * s * (1.f + g * (1.f - s)), d * g * s);
}

void swiglu_bwd(at::Tensor d_act, at::Tensor pre, at::Tensor out) {
  const int64_t n = d_act.numel();
  if (n == 0) return;
  TORCH_CHECK(d_act.is_contiguous() && pre.is_contiguous() && out.is_contiguous(), "swiglu_bwd: contiguous");
  const c10::cuda::CUDAGuard g(pre.device());
  swiglu_bwd_kernel<<<static_cast<int>((n + 255) / 256), 256, 0, cur_stream()>>>(
      reinterpret_cast<const bf16*>(d_act.data_ptr()), reinterpret_cast<const bf16*>(pre.data_ptr()),
      reinterpret_cast<bf16*>(out.data_ptr()), n);
  VLM_LAUNCHED();
}

// ------------------------------------------------------------------ embedding gather / scatter
__global__ void embed_kernel(const int64_t* __restrict__ tok, const bf16* __restrict__ table, bf16* __restrict__ out,
                             int T, int H, int64_t V) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  if (row >= T) return;
  int64_t id = tok[row];
  if (id < 0 || id >= V) id = 0;
  const uint4* src = reinterpret_cast<const uint4*>(table + id * H);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * H);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = src[c];
}

void embed(at::Tensor tokens, at::Tensor table, at::Tensor out) {
  const int T = static_cast<int>(tokens.numel());
  const int H = static_cast<int>(table.size(1));
  if (T == 0) return;
  TORCH_CHECK(tokens.scalar_type() == at::kLong && H % 8 == 0, "embed: int64 tokens, H % 8 == 0");
  const c10::cuda::CUDAGuard g(table.device());
  launch_pdl(embed_kernel, dim3(T), dim3(128), 0, cur_stream(), tokens.data_ptr<int64_t>(),
             reinterpret_cast<const bf16*>(table.data_ptr()), reinterpret_cast<bf16*>(out.data_ptr()), T, H, table.size(0));
}

__global__ void scatter_rows_kernel(bf16* __restrict__ h, const int64_t* __restrict__ rows, const bf16* __restrict__ src,
                                    int R, int H, int add) {
  const int r = blockIdx.x;
  if (r >= R) return;
  bf16* dst = h + rows[r] * H;
  const bf16* s = src + static_cast<int64_t>(r) * H;
  for (int c = threadIdx.x; c < H; c += blockDim.x) dst[c] = add ? f2bf(bf2f(dst[c]) + bf2f(s[c])) : s[c];
}

void scatter_rows(at::Tensor h, at::Tensor rows, at::Tensor src, bool add) {
  const int R = static_cast<int>(rows.numel());
  if (R == 0) return;
  TORCH_CHECK(rows.scalar_type() == at::kLong && src.is_contiguous() && h.is_contiguous(), "scatter_rows: layout");
  const c10::cuda::CUDAGuard g(h.device());
  scatter_rows_kernel<<<R, 128, 0, cur_stream()>>>(reinterpret_cast<bf16*>(h.data_ptr()), rows.data_ptr<int64_t>(),
                                                   reinterpret_cast<const bf16*>(src.data_ptr()), R,
                                                   static_cast<int>(h.size(1)), add ? 1 : 0);
  VLM_LAUNCHED();
}

__global__ void embed_bwd_kernel(const int64_t* __restrict__ tok, const bf16* __restrict__ dh, float* __restrict__ dt,
                                 int T, int H) {
  const int row = blockIdx.x;
  if (row >= T) return;
  const int64_t id = tok[row];
  if (id < 0) return;
  for (int c = threadIdx.x; c < H; c += blockDim.x) atomicAdd(&dt[id * H + c], bf2f(dh[static_cast<int64_t>(row) * H + c]));
}

void embed_bwd(at::Tensor tokens, at::Tensor dh, at::Tensor dtable) {
  const int T = static_cast<int>(tokens.numel());
  if (T == 0) return;
  TORCH_CHECK(dtable.scalar_type() == at::kFloat && dh.is_contiguous(), "embed_bwd: fp32 table grad");
  const c10::cuda::CUDAGuard g(dh.device());
  embed_bwd_kernel<<<T, 256, 0, cur_stream()>>>(tokens.data_ptr<int64_t>(), reinterpret_cast<const bf16*>(dh.data_ptr()),
                                                dtable.data_ptr<float>(), T, static_cast<int>(dh.size(1)));
  VLM_LAUNCHED();
}

// ------------------------------------------------------------------ KV-cache write
// k, v [T, Hkv, D] -> the cache layer (contiguous or paged, KvLayout) at (seq[t], pos[t])
__global__ void kv_write_kernel(const bf16* __restrict__ k, const bf16* __restrict__ v, bf16* __restrict__ kc,
                                bf16* __restrict__ vc, const int64_t* __restrict__ seq, const int64_t* __restrict__ pos,
                                int T, KvLayout lay, int D) {
  const int t = blockIdx.x;
  if (t >= T) return;
  const int64_t s = seq[t], p = pos[t];
  if (p < 0 || p >= lay.cap) return;
  const int Hkv = lay.Hkv;
  for (int i = threadIdx.x; i < Hkv * D / 8; i += blockDim.x) {
    const int h = (i * 8) / D, d = (i * 8) % D;
    const int64_t src = (static_cast<int64_t>(t) * Hkv + h) * D + d;
    const int64_t dst = kv_row(lay, static_cast<int>(s), h, static_cast<int>(p)) * D + d;
    *reinterpret_cast<uint4*>(kc + dst) = *reinterpret_cast<const uint4*>(k + src);
    *reinterpret_cast<uint4*>(vc + dst) = *reinterpret_cast<const uint4*>(v + src);
  }
}

void kv_write(at::Tensor k, at::Tensor v, at::Tensor kc, at::Tensor vc, at::Tensor seq, at::Tensor pos,
              c10::optional<at::Tensor> block_table) {
  const int T = static_cast<int>(k.size(0));
  if (T == 0) return;
  TORCH_CHECK(k.is_contiguous() && v.is_contiguous() && kc.is_contiguous() && vc.is_contiguous(), "kv_write: layout");
  TORCH_CHECK(seq.scalar_type() == at::kLong && pos.scalar_type() == at::kLong, "kv_write: int64 indices");
  const KvLayout lay = kv_layout_of(kc, block_table);
  TORCH_CHECK(k.size(1) == lay.Hkv && vc.sizes() == kc.sizes(), "kv_write: head count / cache shapes");
  const c10::cuda::CUDAGuard g(k.device());
  kv_write_kernel<<<T, 128, 0, cur_stream()>>>(
      reinterpret_cast<const bf16*>(k.data_ptr()), reinterpret_cast<const bf16*>(v.data_ptr()),
      reinterpret_cast<bf16*>(kc.data_ptr()), reinterpret_cast<bf16*>(vc.data_ptr()), seq.data_ptr<int64_t>(),
      pos.data_ptr<int64_t>(), T, lay, static_cast<int>(k.size(2)));
  VLM_LAUNCHED();
}

// ------------------------------------------------------------------ AdamW (optax.adamw semantics)
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, bf16* __restrict__ ph, const float* __restrict__ scale_ptr,
                             int64_t n, float lr, float b1, float b2, float eps, float wd, float bc1, float bc2) {
  const float scale = *scale_ptr;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float gi = g[i] * scale;
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    const float upd = (mi / bc1) / (sqrtf(vi / bc2) + eps) + wd * p[i];
    const float pn = p[i] - lr * upd;
    p[i] = pn;
    if (ph) ph[i] = f2bf(pn);
  }
}

// Same update, 8 elements per thread with 128-bit loads and stores (the parameter units are padded to
// multiples of 128 elements, so every unit takes this path).
__global__ void __launch_bounds__(256) adamw_vec8_kernel(float* __restrict__ p, const float* __restrict__ g,
                                                         float* __restrict__ m, float* __restrict__ v,
                                                         bf16* __restrict__ ph, const float* __restrict__ scale_ptr,
                                                         int64_t n8, float lr, float b1, float b2, float eps, float wd,
                                                         float bc1, float bc2) {
  const float scale = *scale_ptr;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float pv[8], gv[8], mv[8], vv[8];
    const float4* p4 = reinterpret_cast<const float4*>(p) + 2 * i;
    const float4* g4 = reinterpret_cast<const float4*>(g) + 2 * i;
    const float4* m4 = reinterpret_cast<const float4*>(m) + 2 * i;
    const float4* v4 = reinterpret_cast<const float4*>(v) + 2 * i;
    *reinterpret_cast<float4*>(pv) = p4[0];
    *reinterpret_cast<float4*>(pv + 4) = p4[1];
    *reinterpret_cast<float4*>(gv) = g4[0];
    *reinterpret_cast<float4*>(gv + 4) = g4[1];
    *reinterpret_cast<float4*>(mv) = m4[0];
    *reinterpret_cast<float4*>(mv + 4) = m4[1];
    *reinterpret_cast<float4*>(vv) = v4[0];
    *reinterpret_cast<float4*>(vv + 4) = v4[1];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float gi = gv[j] * scale;
      mv[j] = b1 * mv[j] + (1.f - b1) * gi;
      vv[j] = b2 * vv[j] + (1.f - b2) * gi * gi;
      const float upd = (mv[j] / bc1) / (sqrtf(vv[j] / bc2) + eps) + wd * pv[j];
      pv[j] = pv[j] - lr * upd;
    }
    float4* po = reinterpret_cast<float4*>(p) + 2 * i;
    float4* mo = reinterpret_cast<float4*>(m) + 2 * i;
    float4* vo = reinterpret_cast<float4*>(v) + 2 * i;
    po[0] = *reinterpret_cast<float4*>(pv);
    po[1] = *reinterpret_cast<float4*>(pv + 4);
    mo[0] = *reinterpret_cast<float4*>(mv);
    mo[1] = *reinterpret_cast<float4*>(mv + 4);
    vo[0] = *reinterpret_cast<float4*>(vv);
    vo[1] = *reinterpret_cast<float4*>(vv + 4);
    if (ph)
      reinterpret_cast<uint4*>(ph)[i] = make_uint4(pack_bf16x2(pv[0], pv[1]), pack_bf16x2(pv[2], pv[3]),
                                                   pack_bf16x2(pv[4], pv[5]), pack_bf16x2(pv[6], pv[7]));
  }
}

void adamw(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, at::Tensor ph, at::Tensor scale, double lr, double b1,
           double b2, double eps, double wd, int64_t step) {
  const int64_t n = p.numel();
  if (n == 0) return;
  TORCH_CHECK(p.scalar_type() == at::kFloat && g.scalar_type() == at::kFloat && p.is_contiguous() && g.is_contiguous(),
              "adamw: fp32 contiguous");
  const c10::cuda::CUDAGuard gd(p.device());
  const float bc1 = static_cast<float>(1.0 - std::pow(b1, static_cast<double>(step)));
  const float bc2 = static_cast<float>(1.0 - std::pow(b2, static_cast<double>(step)));
  auto aligned = [](const at::Tensor& t) { return reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0; };
  const bool has_ph = ph.defined() && ph.numel();
  if (n % 8 == 0 && aligned(p) && aligned(g) && aligned(m) && aligned(v) && (!has_ph || aligned(ph)) &&
      m.is_contiguous() && v.is_contiguous() && (!has_ph || ph.is_contiguous())) {
    const int blocks = static_cast<int>(std::min<int64_t>((n / 8 + 255) / 256, num_sms(p.device().index()) * 8));
    adamw_vec8_kernel<<<blocks, 256, 0, cur_stream()>>>(
        p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
        has_ph ? reinterpret_cast<bf16*>(ph.data_ptr()) : nullptr, scale.data_ptr<float>(), n / 8,
        static_cast<float>(lr), static_cast<float>(b1), static_cast<float>(b2), static_cast<float>(eps),
        static_cast<float>(wd), bc1, bc2);
    VLM_LAUNCHED();
    return;
  }
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, num_sms(p.device().index()) * 8));
  adamw_kernel<<<blocks, 256, 0, cur_stream()>>>(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(),
                                                 v.data_ptr<float>(),
                                                 ph.defined() && ph.numel() ? reinterpret_cast<bf16*>(ph.data_ptr()) : nullptr,
                                                 scale.data_ptr<float>(), n, static_cast<float>(lr), static_cast<float>(b1),
                                                 static_cast<float>(b2), static_cast<float>(eps), static_cast<float>(wd),
                                                 bc1, bc2);
  VLM_LAUNCHED();
}

// ------------------------------------------------------------------ sum of squares (fp32 accumulate)
template <typename T>
__global__ void sq_norm_kernel(const T* __restrict__ x, int64_t n, float* __restrict__ out) {
  float s = 0.f;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float f = static_cast<float>(x[i]);
    s += f * f;
  }
  s = warp_sum(s);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) atomicAdd(out, t);
  }
}

// fp32 input, 16-byte aligned, n % 16 == 0: four float4 loads in flight per thread per iteration (the
// scalar loop above kept one 4-byte load in flight and read gradients at half the HBM rate).
__global__ void sq_norm_vec_kernel(const float4* __restrict__ x, int64_t n16, float* __restrict__ out) {
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n16;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float4 a = __ldcs(x + 4 * i), b = __ldcs(x + 4 * i + 1), c = __ldcs(x + 4 * i + 2),
                 d = __ldcs(x + 4 * i + 3);
    s0 += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
    s1 += b.x * b.x + b.y * b.y + b.z * b.z + b.w * b.w;
    s2 += c.x * c.x + c.y * c.y + c.z * c.z + c.w * c.w;
    s3 += d.x * d.x + d.y * d.y + d.z * d.z + d.w * d.w;
  }
  float s = warp_sum((s0 + s1) + (s2 + s3));
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) atomicAdd(out, t);
  }
}

void sq_norm_acc(at::Tensor x, at::Tensor out) {
  const int64_t n = x.numel();
  if (n == 0) return;
  TORCH_CHECK(x.is_contiguous() && out.scalar_type() == at::kFloat, "sq_norm: contiguous input, fp32 out");
  const c10::cuda::CUDAGuard g(x.device());
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, num_sms(x.device().index()) * 4));
  if (x.scalar_type() == at::kFloat && n % 16 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0) {
    const int vblocks = static_cast<int>(std::min<int64_t>((n / 16 + 255) / 256, num_sms(x.device().index()) * 4));
    sq_norm_vec_kernel<<<vblocks, 256, 0, cur_stream()>>>(reinterpret_cast<const float4*>(x.data_ptr<float>()),
                                                          n / 16, out.data_ptr<float>());
  } else if (x.scalar_type() == at::kFloat)
    sq_norm_kernel<float><<<blocks, 256, 0, cur_stream()>>>(x.data_ptr<float>(), n, out.data_ptr<float>());
  else
    sq_norm_kernel<__nv_bfloat16><<<blocks, 256, 0, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), n, out.data_ptr<float>());
  VLM_LAUNCHED();
}

// ------------------------------------------------------------------ uint8 image -> patch rows
// images [N, H, W, 3] uint8 -> rows [N*gh*gw, 3*Tp*P*P] bf16, rows in merge-window order,
// row layout (c, t, py, px); the single frame is repeated over the temporal patch.
__global__ void patchify_kernel(const uint8_t* __restrict__ img, const float* __restrict__ ms, bf16* __restrict__ out,
                                int N, int H, int W, int P, int Tp, int merge) {
  const int gh = H / P, gw = W / P;
  const int row = blockIdx.x;  // over N*gh*gw
  const int per_img = gh * gw;
  const int n = row / per_img, r = row % per_img;
  const int wb_count = gw / merge;
  const int blk = r / (merge * merge), in = r % (merge * merge);
  const int hb = blk / wb_count, wb = blk % wb_count;
  const int py0 = (hb * merge + in / merge) * P, px0 = (wb * merge + in % merge) * P;
  const int cols = 3 * Tp * P * P;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    const int ch = c / (Tp * P * P);
    const int rem = c % (P * P);
    const int y = py0 + rem / P, x = px0 + rem % P;
    const float val = static_cast<float>(img[((static_cast<int64_t>(n) * H + y) * W + x) * 3 + ch]) * (1.f / 255.f);
    out[static_cast<int64_t>(row) * cols + c] = f2bf((val - ms[ch]) / ms[3 + ch]);
  }
}

void patchify(at::Tensor images, at::Tensor ms, at::Tensor out, int64_t patch, int64_t temporal, int64_t merge) {
  TORCH_CHECK(images.scalar_type() == at::kByte && images.is_contiguous() && images.size(3) == 3, "patchify: uint8 NHWC");
  const int N = static_cast<int>(images.size(0)), H = static_cast<int>(images.size(1)), W = static_cast<int>(images.size(2));
  const int rows = N * (H / static_cast<int>(patch)) * (W / static_cast<int>(patch));
  if (rows == 0) return;
  const c10::cuda::CUDAGuard g(images.device());
  patchify_kernel<<<rows, 256, 0, cur_stream()>>>(images.data_ptr<uint8_t>(), ms.data_ptr<float>(),
                                                  reinterpret_cast<bf16*>(out.data_ptr()), N, H, W, static_cast<int>(patch),
                                                  static_cast<int>(temporal), static_cast<int>(merge));
  VLM_LAUNCHED();
}

}  // namespace vlm

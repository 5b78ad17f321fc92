// Decode consumers that run inside the stream-K GEMM that produces their partial sums.
//
// A decode-step GEMM (M = batch rows) writes fp32 partial sums per (tile, k-range) slot.  Instead of
// handing them to a separate consumer kernel, every CTA of the GEMM waits at a grid-wide barrier after
// its partial stores and then takes a share of the consumer's work:
//   DEC_QKV      sum + bias -> per-head RMSNorm of q/k (optional) -> MRoPE -> q out, k/v into the cache
//   DEC_RESNORM  sum + residual -> h (bf16) -> RMSNorm(h) * w -> hn (bf16)
//   DEC_SWIGLU   sum -> silu(gate) * up of interleaved (gate, up) columns
// which removes one launch (and its dependency latency) per GEMM of the decode loop.
//
// The GEMM is launched cooperatively with one CTA per SM, so all CTAs are resident and the barrier
// cannot wait for a CTA that never runs.  The barrier is self-resetting (arrival count + generation),
// so a CUDA graph can replay it, and bounded: after kWaitCycles a waiter records kErrTimeoutFlag and the
// CTA skips the consumer.
#pragma once

#include "common.cuh"
#include "streamk.cuh"

namespace vlm {

enum DecConsumer : int { DEC_NONE = 0, DEC_QKV = 1, DEC_RESNORM = 2, DEC_SWIGLU = 3 };

struct DecArgs {
  // DEC_QKV
  const __nv_bfloat16* bias;
  const __nv_bfloat16* qw;  // null: rotation only (no q/k RMSNorm)
  const __nv_bfloat16* kw;
  const int* lengths;
  const int64_t* delta;
  const float* inv_freq;
  __nv_bfloat16* q;
  __nv_bfloat16* kc;
  __nv_bfloat16* vc;
  int nq, nkv, Tmax, head_dim;
  // DEC_RESNORM
  const __nv_bfloat16* res;
  const __nv_bfloat16* nw;
  __nv_bfloat16* h_out;
  __nv_bfloat16* hn_out;
  // DEC_SWIGLU
  __nv_bfloat16* act;
  float eps;
};

VLM_DEV unsigned dec_ld_acquire(const unsigned* a) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}

// Grid-wide barrier over all CTAs of the launch; bar[0] = arrivals, bar[1] = generation.  Every thread
// of the CTA calls it; returns false (on every thread) when the wait ran out.
VLM_DEV bool dec_grid_sync(unsigned* bar, int* err, int* flag_smem) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned gen = dec_ld_acquire(bar + 1);
    __threadfence();
    bool ok = true;
    if (atomicAdd(bar, 1u) == gridDim.x - 1) {
      atomicExch(bar, 0u);
      __threadfence();
      asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar + 1) : "memory");
    } else {
      const long long t0 = clock64();
      while (dec_ld_acquire(bar + 1) == gen) {
        if (clock64() - t0 > kWaitCycles) {
          atomicCAS(err, 0, kErrTimeoutFlag);
          ok = false;
          break;
        }
      }
    }
    __threadfence();
    *flag_smem = ok;
  }
  __syncthreads();
  return *flag_smem != 0;
}

VLM_DEV void dec_store8(__nv_bfloat16* dst, const float (&v)[8]) {
  *reinterpret_cast<uint4*>(dst) =
      make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
}

// q/k/v consumer: groups of TPH = D/8 lanes own one (row, head) item; a warp's groups walk the items
// together so the per-head shuffles always see the whole warp.
template <int D>
VLM_DEV void dec_qkv_part(const float* __restrict__ ws, const SkMeta& m, const DecArgs& a) {
  constexpr int TPH = D / 8, GPW = 32 / TPH;
  const int lane = threadIdx.x & 31, t = lane % TPH;
  const int heads = a.nq + 2 * a.nkv;
  const long long items = static_cast<long long>(m.M) * heads;
  const long long warps_total = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long base = (static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * GPW;
       base < items; base += warps_total * GPW) {
    const long long item = base + lane / TPH;
    const bool valid = item < items;
    const int row = valid ? static_cast<int>(item / heads) : 0;
    const int head = valid ? static_cast<int>(item % heads) : 0;
    const int col = head * D + t * 8;
    float x[8];
    if (valid) {
      sk_sum8(ws, m, row, col, x);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = bf2f(f2bf(x[i] + (a.bias && valid ? bf2f(a.bias[col + i]) : 0.f)));
    const bool is_v = head >= a.nq + a.nkv, is_q = head < a.nq;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += x[i] * x[i];
#pragma unroll
    for (int off = TPH / 2; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const bool norm = a.qw != nullptr;
    const float r = norm ? rsqrtf(ss / D + a.eps) : 1.f;
    const __nv_bfloat16* wt = is_q ? a.qw : a.kw;
    float xn[8], y[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) xn[i] = (is_v || !norm) ? x[i] : x[i] * r * bf2f(wt[t * 8 + i]);
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = __shfl_xor_sync(0xffffffffu, xn[i], TPH / 2);
    if (!valid) continue;
    const int len = a.lengths[row];
    if (is_v) {
      dec_store8(a.vc + ((static_cast<int64_t>(row) * a.nkv + (head - a.nq - a.nkv)) * a.Tmax + len) * D + t * 8, x);
      continue;
    }
    const float pos = static_cast<float>(static_cast<int64_t>(len) + a.delta[row]);
    const bool first_half = t < TPH / 2;
    float out[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float s, c;
      sincosf(pos * a.inv_freq[(t % (TPH / 2)) * 8 + i], &s, &c);
      out[i] = first_half ? xn[i] * c - y[i] * s : xn[i] * c + y[i] * s;
    }
    if (is_q)
      dec_store8(a.q + (static_cast<int64_t>(row) * a.nq + head) * D + t * 8, out);
    else
      dec_store8(a.kc + ((static_cast<int64_t>(row) * a.nkv + (head - a.nq)) * a.Tmax + len) * D + t * 8, out);
  }
}

// residual + RMSNorm consumer: one CTA per row (rows strided over the grid); H <= 8 * blockDim * CH.
template <int CH>
VLM_DEV void dec_resnorm_part(const float* __restrict__ ws, const SkMeta& m, const DecArgs& a, float* red) {
  const int H = m.N;
  const int nthr = blockDim.x, tid = threadIdx.x;
  for (int row = blockIdx.x; row < m.M; row += gridDim.x) {
    float x[CH][8];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int col = (tid + c * nthr) * 8;
      if (col < H) {
        sk_sum8(ws, m, row, col, x[c]);
        const uint4 rv = *reinterpret_cast<const uint4*>(a.res + static_cast<int64_t>(row) * H + col);
        const uint32_t u[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack_bf16x2(u[j]);
          x[c][2 * j] = bf2f(f2bf(x[c][2 * j] + f.x));
          x[c][2 * j + 1] = bf2f(f2bf(x[c][2 * j + 1] + f.y));
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += x[c][i] * x[c][i];
        dec_store8(a.h_out + static_cast<int64_t>(row) * H + col, x[c]);
      }
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    if (tid < 32) {
      float v = tid < (nthr + 31) / 32 ? red[tid] : 0.f;
      v = warp_sum(v);
      if (tid == 0) red[32] = v;
    }
    __syncthreads();
    const float r = rsqrtf(red[32] / H + a.eps);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int col = (tid + c * nthr) * 8;
      if (col < H) {
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = bf2f(f2bf(x[c][i] * r)) * bf2f(a.nw[col + i]);
        dec_store8(a.hn_out + static_cast<int64_t>(row) * H + col, o);
      }
    }
    __syncthreads();  // red[] is reused by the next row
  }
}

// SwiGLU consumer: grid-stride over (row, 8 columns) of the interleaved gate/up partials.
VLM_DEV void dec_swiglu_part(const float* __restrict__ ws, const SkMeta& m, const DecArgs& a) {
  const int N = m.N, per_row = N / 8;
  const long long items = static_cast<long long>(m.M) * per_row;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < items;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(i / per_row), col = static_cast<int>(i % per_row) * 8;
    float x[8];
    sk_sum8(ws, m, row, col, x);
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float g = bf2f(f2bf(x[2 * j])), u = bf2f(f2bf(x[2 * j + 1]));
      o[j] = g / (1.f + __expf(-g)) * u;
    }
    *reinterpret_cast<uint2*>(a.act + static_cast<int64_t>(row) * (N / 2) + col / 2) =
        make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
  }
}

}  // namespace vlm

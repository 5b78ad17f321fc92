// Decode-step kernels that consume the stream-K partial sums of the skinny (M = batch) GEMMs and
// fuse the memory-bound work that follows each of them:
//   dec_qkv            sum partials + bias -> per-head RMSNorm of q/k -> MRoPE -> q out, k/v into the KV cache
//   dec_residual_norm  sum partials + residual -> h (bf16) -> RMSNorm(h) -> hn (bf16)
//   dec_swiglu         sum partials -> silu(gate) * up
// so a decoder layer is 4 GEMMs + 3 of these + attention, with no separate reduction launches.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "kv_layout.cuh"
#include "host_utils.h"
#include "peer.cuh"
#include "streamk.cuh"
#include "vlm_ops.h"

namespace vlm {

using bf16 = __nv_bfloat16;

static SkMeta meta_of(const std::vector<int64_t>& v) {
  TORCH_CHECK(v.size() == 8, "stream-K meta must have 8 entries");
  return SkMeta{static_cast<int>(v[0]), static_cast<int>(v[1]), static_cast<int>(v[2]), static_cast<int>(v[3]),
                static_cast<int>(v[4]), static_cast<int>(v[5]), static_cast<int>(v[6]), static_cast<int>(v[7])};
}

VLM_DEV void store8(bf16* dst, const float (&v)[8]) {
  *reinterpret_cast<uint4*>(dst) =
      make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
}

// One CTA per token row; thread i owns qkv columns [8i, 8i+8).  TPH = D/8 threads per head.
template <int D>
__global__ void dec_qkv_kernel(const float* __restrict__ ws, SkMeta m, const bf16* __restrict__ bias,
                               const bf16* __restrict__ qw, const bf16* __restrict__ kw, const int* __restrict__ lengths,
                               const int64_t* __restrict__ delta, const float* __restrict__ inv_freq,
                               bf16* __restrict__ q, bf16* __restrict__ kc, bf16* __restrict__ vc, int nq, int nkv,
                               KvLayout lay, float eps, L2Prefetch pf) {
  constexpr int TPH = D / 8;
  l2_prefetch_share(pf);
  const int row = blockIdx.x, tid = threadIdx.x;
  const int head = tid / TPH, t = tid % TPH;
  const int col = tid * 8;
  // The cache lengths, rotary offsets and bias were written before the previous kernel (the GEMM whose
  // partials this kernel sums) started, so they are read before the dependency wait.
  const int len = lengths[row];
  const int64_t dl = delta[row];
  float bv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) bv[i] = bias ? bf2f(bias[col + i]) : 0.f;
  pdl_wait();
  pdl_trigger();
  float x[8];
  sk_sum8(ws, m, row, col, x);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = bf2f(f2bf(x[i] + bv[i]));
  const bool is_v = head >= nq + nkv;
  const bool is_q = head < nq;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += x[i] * x[i];
#pragma unroll
  for (int off = TPH / 2; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const bool norm = qw != nullptr;  // no q/k RMSNorm (Qwen2.5-style attention): rotate only
  const float r = norm ? rsqrtf(ss / D + eps) : 1.f;
  const bf16* wt = is_q ? qw : kw;
  float xn[8], y[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) xn[i] = (is_v || !norm) ? x[i] : x[i] * r * bf2f(wt[t * 8 + i]);
#pragma unroll
  for (int i = 0; i < 8; ++i) y[i] = __shfl_xor_sync(0xffffffffu, xn[i], TPH / 2);
  if (is_v) {
    if (len < lay.cap) store8(vc + kv_row(lay, row, head - nq - nkv, len) * D + t * 8, x);
    return;
  }
  const float pos = static_cast<float>(static_cast<int64_t>(len) + dl);
  const bool first_half = t < TPH / 2;
  float out[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float s, c;
    sincosf(pos * inv_freq[(t % (TPH / 2)) * 8 + i], &s, &c);
    out[i] = first_half ? xn[i] * c - y[i] * s : xn[i] * c + y[i] * s;
  }
  if (is_q)
    store8(q + (static_cast<int64_t>(row) * nq + head) * D + t * 8, out);
  else if (len < lay.cap)
    store8(kc + kv_row(lay, row, head - nq, len) * D + t * 8, out);
}

// One CTA per row; thread i owns columns [8i, 8i+8).
__global__ void dec_resnorm_kernel(const float* __restrict__ ws, SkMeta m, const bf16* __restrict__ res,
                                   const bf16* __restrict__ w, bf16* __restrict__ h_out, bf16* __restrict__ hn_out,
                                   int H, float eps, L2Prefetch pf) {
  __shared__ float red[32];
  l2_prefetch_share(pf);
  const int row = blockIdx.x, col = threadIdx.x * 8;
  // The residual row and the norm weight were written before the previous kernel (the GEMM whose partials
  // this kernel sums) started, so they are read before the dependency wait.
  uint4 rv = make_uint4(0, 0, 0, 0), wv = make_uint4(0, 0, 0, 0);
  if (col < H) {
    rv = *reinterpret_cast<const uint4*>(res + static_cast<int64_t>(row) * H + col);
    wv = *reinterpret_cast<const uint4*>(w + col);
  }
  pdl_wait();
  pdl_trigger();
  float x[8];
  float ss = 0.f;
  if (col < H) {
    sk_sum8(ws, m, row, col, x);
    const uint32_t u[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(u[j]);
      x[2 * j] = bf2f(f2bf(x[2 * j] + f.x));
      x[2 * j + 1] = bf2f(f2bf(x[2 * j + 1] + f.y));
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += x[i] * x[i];
    store8(h_out + static_cast<int64_t>(row) * H + col, x);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x + 31) / 32 ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  if (col < H) {
    const float r = rsqrtf(red[0] / H + eps);
    const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
    float o[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(wu[j]);
      o[2 * j] = bf2f(f2bf(x[2 * j] * r)) * f.x;
      o[2 * j + 1] = bf2f(f2bf(x[2 * j + 1] * r)) * f.y;
    }
    store8(hn_out + static_cast<int64_t>(row) * H + col, o);
  }
}

__global__ void dec_swiglu_kernel(const float* __restrict__ ws, SkMeta m, bf16* __restrict__ act, int N, L2Prefetch pf) {
  l2_prefetch_share(pf);
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.y;
  const int col = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (col >= N) return;
  float x[8];
  sk_sum8(ws, m, row, col, x);
  float o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float g = bf2f(f2bf(x[2 * j])), u = bf2f(f2bf(x[2 * j + 1]));
    o[j] = g / (1.f + __expf(-g)) * u;
  }
  *reinterpret_cast<uint2*>(act + static_cast<int64_t>(row) * (N / 2) + col / 2) =
      make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
}

at::Tensor dec_qkv(at::Tensor ws, std::vector<int64_t> meta, at::Tensor bias, at::Tensor qw, at::Tensor kw,
                   at::Tensor lengths, at::Tensor delta, at::Tensor inv_freq, at::Tensor kc, at::Tensor vc, int64_t nq,
                   int64_t nkv, double eps, c10::optional<at::Tensor> prefetch,
                   c10::optional<at::Tensor> block_table) {
  const SkMeta m = meta_of(meta);
  const L2Prefetch pf = l2_prefetch_of<L2Prefetch>(prefetch);
  const int D = static_cast<int>(kc.size(-1));
  const KvLayout lay = kv_layout_of(kc, block_table);
  TORCH_CHECK(lay.Hkv == nkv && vc.sizes() == kc.sizes(), "dec_qkv: cache heads / shapes");
  TORCH_CHECK(m.N == (nq + 2 * nkv) * D, "dec_qkv: width mismatch");
  TORCH_CHECK(lengths.scalar_type() == at::kInt && delta.scalar_type() == at::kLong, "dec_qkv: int32 lengths, int64 deltas");
  TORCH_CHECK(kc.is_contiguous() && vc.is_contiguous(), "dec_qkv: contiguous cache layer");
  const c10::cuda::CUDAGuard g(ws.device());
  at::Tensor q = at::empty({m.M, nq, D}, kc.options());
  const int threads = static_cast<int>((nq + 2 * nkv) * D / 8);
  TORCH_CHECK(threads <= 1024, "dec_qkv: too many heads for one CTA");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto args = [&](auto kern) {
    launch_pdl(kern, dim3(m.M), dim3(threads), 0, st, ws.data_ptr<float>(), m,
               bias.defined() && bias.numel() ? reinterpret_cast<const bf16*>(bias.data_ptr()) : nullptr,
               qw.defined() && qw.numel() ? reinterpret_cast<const bf16*>(qw.data_ptr()) : nullptr,
               kw.defined() && kw.numel() ? reinterpret_cast<const bf16*>(kw.data_ptr()) : nullptr,
               lengths.data_ptr<int>(), delta.data_ptr<int64_t>(), inv_freq.data_ptr<float>(),
               reinterpret_cast<bf16*>(q.data_ptr()), reinterpret_cast<bf16*>(kc.data_ptr()),
               reinterpret_cast<bf16*>(vc.data_ptr()), static_cast<int>(nq), static_cast<int>(nkv), lay,
               static_cast<float>(eps), pf);
  };
  if (D == 128)
    args(dec_qkv_kernel<128>);
  else if (D == 64)
    args(dec_qkv_kernel<64>);
  else if (D == 32)
    args(dec_qkv_kernel<32>);
  else
    TORCH_CHECK(false, "dec_qkv: unsupported head_dim ", D);
  return q;
}

std::tuple<at::Tensor, at::Tensor> dec_residual_norm(at::Tensor ws, std::vector<int64_t> meta, at::Tensor residual,
                                                     at::Tensor w, double eps, c10::optional<at::Tensor> prefetch) {
  const SkMeta m = meta_of(meta);
  TORCH_CHECK(residual.is_contiguous() && residual.size(0) == m.M && residual.size(1) == m.N, "dec_residual_norm: shape");
  TORCH_CHECK(m.N % 8 == 0 && m.N / 8 <= 1024, "dec_residual_norm: width");
  const c10::cuda::CUDAGuard g(ws.device());
  at::Tensor h = at::empty_like(residual), hn = at::empty_like(residual);
  const int threads = ((m.N / 8 + 31) / 32) * 32;
  launch_pdl(dec_resnorm_kernel, dim3(m.M), dim3(threads), 0, at::cuda::getCurrentCUDAStream(), ws.data_ptr<float>(), m,
             reinterpret_cast<const bf16*>(residual.data_ptr()), reinterpret_cast<const bf16*>(w.data_ptr()),
             reinterpret_cast<bf16*>(h.data_ptr()), reinterpret_cast<bf16*>(hn.data_ptr()), m.N, static_cast<float>(eps),
             l2_prefetch_of<L2Prefetch>(prefetch));
  return {h, hn};
}

at::Tensor dec_swiglu(at::Tensor ws, std::vector<int64_t> meta, c10::optional<at::Tensor> prefetch) {
  const SkMeta m = meta_of(meta);
  TORCH_CHECK(m.N % 16 == 0, "dec_swiglu: width must be a multiple of 16");
  const c10::cuda::CUDAGuard g(ws.device());
  at::Tensor act = at::empty({m.M, m.N / 2}, ws.options().dtype(at::kBFloat16));
  const dim3 grid((m.N / 8 + 255) / 256, m.M);
  launch_pdl(dec_swiglu_kernel, grid, dim3(256), 0, at::cuda::getCurrentCUDAStream(), ws.data_ptr<float>(), m,
             reinterpret_cast<bf16*>(act.data_ptr()), m.N, l2_prefetch_of<L2Prefetch>(prefetch));
  return act;
}


// ------------------------------------------------------------------ tensor-parallel decode consumers
// Row-parallel GEMMs (o_proj, down_proj) leave each rank with a partial sum of the full [B, H] output.
// dec_resnorm_tp_kernel all-reduces it over NVLink inside the consumer, with no fence and no separate
// flag on the critical path.  Every value travels with the step's tag in one 8-byte word: fp32 bits in
// the low half, the low 32 bits of the device-side step epoch in the high half.  CTA `row` (1) sums this
// rank's stream-K slots of its row and stores the tagged words straight into slot `rank` of every
// rank's buffer ([W][max_batch][H] words per point), (2) polls its own buffer until every rank's word of
// its columns carries the tag (bounded), (3) adds the ranks' values in rank order (identical on every
// rank), then the residual, and applies the RMSNorm.  An aligned 8-byte store is single-copy atomic, so
// a reader sees a word whole: old tag (keep polling) or new tag with its value.  Critical path: one
// one-way NVLink store instead of a fence, a flag and a remote read.  A rank overwrites a peer's slot of
// a point one decode step later, after it has seen that peer's words of a later point, which the peer
// stores only after its kernel for this point (and its reads) completed.
__global__ void tp_step_begin_kernel(unsigned long long* epoch) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) epoch[0] += 1ull;
}

VLM_DEV unsigned long long tag_word(float v, unsigned tag) {
  return (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
}
VLM_DEV void st_tagged2(unsigned long long* a, unsigned long long w0, unsigned long long w1) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(a), "l"(w0), "l"(w1) : "memory");
}
VLM_DEV void ld_tagged2(const unsigned long long* a, unsigned long long& w0, unsigned long long& w1) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(a) : "memory");
}

__global__ void dec_resnorm_tp_kernel(const float* __restrict__ ws, SkMeta m, const bf16* __restrict__ res,
                                      const bf16* __restrict__ w, bf16* __restrict__ h_out, bf16* __restrict__ hn_out,
                                      int H, float eps, PeerTable slots, int max_batch,
                                      const unsigned long long* __restrict__ epoch_ptr, int rank, int W, int* err) {
  __shared__ float red[32];
  __shared__ int ok;
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x, col = threadIdx.x * 8;
  const unsigned tag = static_cast<unsigned>(*epoch_ptr);
  if (threadIdx.x == 0) ok = 1;
  float x[8];
  if (col < H) {
    sk_sum8(ws, m, row, col, x);
    const int64_t off = (static_cast<int64_t>(rank) * max_batch + row) * H + col;
    for (int p = 0; p < W; ++p) {
      unsigned long long* dst = reinterpret_cast<unsigned long long*>(slots.p[p]) + off;
#pragma unroll
      for (int i = 0; i < 8; i += 2) st_tagged2(dst + i, tag_word(x[i], tag), tag_word(x[i + 1], tag));
    }
  }
  __syncthreads();  // ok = 1 is seen before any thread can clear it
  float sum[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) sum[i] = 0.f;
  if (col < H) {
    const unsigned long long* mine = reinterpret_cast<const unsigned long long*>(slots.p[rank]);
    const long long t0 = clock64();
    bool good = true;
    for (int p = 0; p < W && good; ++p) {
      if (p == rank) {
#pragma unroll
        for (int i = 0; i < 8; ++i) sum[i] += x[i];
        continue;
      }
      const unsigned long long* src = mine + (static_cast<int64_t>(p) * max_batch + row) * H + col;
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        unsigned long long w0, w1;
        ld_tagged2(src + i, w0, w1);
        while (static_cast<unsigned>(w0 >> 32) != tag || static_cast<unsigned>(w1 >> 32) != tag) {
          if (clock64() - t0 > kPeerWait) {
            atomicCAS(err, 0, kErrTimeoutPeer);
            good = false;
            break;
          }
          ld_tagged2(src + i, w0, w1);
        }
        sum[i] += __uint_as_float(static_cast<unsigned>(w0));
        sum[i + 1] += __uint_as_float(static_cast<unsigned>(w1));
      }
    }
    if (!good) ok = 0;
  }
  __syncthreads();
  if (!ok) return;
  float ss = 0.f;
  const int64_t off = static_cast<int64_t>(row) * H + col;
  if (col < H) {
    const uint4 rv = *reinterpret_cast<const uint4*>(res + off);
    const uint32_t u[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(u[j]);
      x[2 * j] = bf2f(f2bf(sum[2 * j] + f.x));
      x[2 * j + 1] = bf2f(f2bf(sum[2 * j + 1] + f.y));
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += x[i] * x[i];
    store8(h_out + off, x);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x + 31) / 32 ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  if (col < H) {
    const float r = rsqrtf(red[0] / H + eps);
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = bf2f(f2bf(x[i] * r)) * bf2f(w[col + i]);
    store8(hn_out + off, o);
  }
}

void tp_step_begin(int64_t epoch_ptr, int64_t device) {
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  launch_pdl(tp_step_begin_kernel, dim3(1), dim3(32), 0, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<unsigned long long*>(epoch_ptr));
}

// h = residual + all-reduce over ranks of this rank's partials; hn = rms_norm(h) * w.  `slots` are the
// per-rank addresses of the IPC-shared word buffer of this point ([W][max_batch][H] tagged 8-byte words).
std::tuple<at::Tensor, at::Tensor> dec_residual_norm_tp(at::Tensor ws, std::vector<int64_t> meta, at::Tensor res,
                                                        at::Tensor w, double eps, std::vector<int64_t> slots,
                                                        int64_t slot_off_bytes, int64_t max_batch, int64_t epoch_ptr,
                                                        int64_t rank) {
  const SkMeta m = meta_of(meta);
  const int H = m.N;
  const int W = static_cast<int>(slots.size());
  TORCH_CHECK(H % 8 == 0 && H / 8 <= 1024, "dec_residual_norm_tp: H must be a multiple of 8 and <= 8192");
  TORCH_CHECK(rank >= 0 && rank < W && m.M <= max_batch, "dec_residual_norm_tp: rank / batch");
  TORCH_CHECK(slot_off_bytes % 16 == 0, "dec_residual_norm_tp: slot buffer alignment");
  const c10::cuda::CUDAGuard g(ws.device());
  at::Tensor h = at::empty({m.M, H}, res.options());
  at::Tensor hn = at::empty({m.M, H}, res.options());
  const int threads = ((H / 8 + 31) / 32) * 32;
  launch_pdl(dec_resnorm_tp_kernel, dim3(m.M), dim3(threads), 0, at::cuda::getCurrentCUDAStream(),
             ws.data_ptr<float>(), m, reinterpret_cast<const bf16*>(res.data_ptr()),
             reinterpret_cast<const bf16*>(w.data_ptr()), reinterpret_cast<bf16*>(h.data_ptr()),
             reinterpret_cast<bf16*>(hn.data_ptr()), H, static_cast<float>(eps), make_peer_table(slots, slot_off_bytes),
             static_cast<int>(max_batch), reinterpret_cast<const unsigned long long*>(epoch_ptr),
             static_cast<int>(rank), W, err_word(ws.device().index()));
  return {h, hn};
}

}  // namespace vlm

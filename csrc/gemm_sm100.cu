// Persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   D[M,N] = alpha * A[M,K] . B[N,K]^T   (+bias[N]) (+residual[M,N]) (activation) (+= D when accumulating)
//
// * A and B are bf16 in either K-major or MN-major layout (the latter lets the
//   backward GEMMs dX = dY.W and dW = dY^T.X read activations and weights in
//   place, without transposes).
// * Tiles are 128 x BN x 64 (BN = 128 or 256).  Operands are staged by TMA
//   (128-byte swizzle) into a STAGES-deep shared-memory ring guarded by
//   mbarriers; one elected thread issues tcgen05.mma (UMMA 128xBNx16) into a
//   double-buffered TMEM accumulator; four epilogue warps drain TMEM with
//   tcgen05.ld while the next tile's MMAs run.
// * Warp roles: 0 = TMA producer, 1 = MMA issuer (+TMEM owner), 2..5 = epilogue.
// * Grid = min(#tiles, #SMs) CTAs, one per SM; tiles are walked in groups of
//   16 M-tiles so concurrently running CTAs share B tiles in L2.
// * Every wait is bounded (see common.cuh); on timeout the kernel records an
//   error code, drains its own in-flight TMA copies and MMAs, frees TMEM and exits.
// * GATHER variant (FSDP with sharded parameters): B is a weight whose rows are
//   spread over the ranks' parameter shards.  Two extra copy warps per CTA pull
//   64-row chunks from every rank's shard (plain peer loads over NVLink) into
//   the local buffer the B tensor map covers, 16 KB pieces claimed from a
//   global queue; the TMA producer waits on a chunk's arrival count before it
//   loads from that chunk, so the all-gather overlaps the MMAs tile by tile.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "host_utils.h"
#include "peer.cuh"
#include "dec_fused.cuh"
#include "vlm_ops.h"
#include "streamk.cuh"

namespace vlm {

using bf16_t = __nv_bfloat16;

struct DecFuse {
  int consumer;
  DecArgs args;
};

enum Epi : int {
  EPI_STORE = 0, EPI_SWIGLU = 1, EPI_GELU_TANH = 2, EPI_GELU_ERF = 3, EPI_VOCAB_STATS = 4, EPI_VOCAB_GRAD = 5,
  // D [M, 2N] = SwiGLU backward of the product (= dL/d act) with aux = the forward's interleaved (gate, up)
  EPI_SWIGLU_BWD = 6,
  // no D: per (row, N-tile) the topk largest products (value desc, index asc) -> part / cand_i [M][tiles_n][topk]
  EPI_TOPK = 7
};
constexpr int kTopkMax = 16;  // top-k epilogue: at most this many candidates per (row, tile)

struct GemmParams {
  int M, N, K;
  void* D;
  long long ldd;
  int d_f32;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* residual;
  long long ldr;
  __nv_bfloat16* aux;
  long long ld_aux;
  float alpha;
  int epi;
  int accumulate;
  int tiles_m, tiles_n;
  int* err;
  // vocab epilogues (per-row data of the fused lm_head -> log-softmax)
  const int64_t* targets;
  const float* row_lse;
  const float* row_ent;
  const float* g_lp;
  const float* g_ent;
  float* part;  // [M, tiles_n, 4] partial (max, sum exp, sum exp*z, target logit); EPI_TOPK: candidate values
  int* cand_i;  // EPI_TOPK: candidate indices [M, tiles_n, topk]
  int topk;
  // split-K: tile t -> (mn tile = t / splits, split = t % splits); each split stores raw fp32
  // partial sums to ws[split] ([M, N] row-major) and splitk_reduce applies the epilogue.
  int splits;
  int kb_per_split;
  float* ws;
  // stream-K: CTA c owns the contiguous (tile, k-block) units [c*U/G, (c+1)*U/G), U = tiles*kb_count
  int streamk;
  int sk_grid;  // grid size of the stream-K launch
  int bn;
  int b_prefetch;  // B may be loaded before pdl_wait (B is a weight no earlier kernel of the step writes)
  // optional phase timestamps (%globaltimer, ns) per CTA: [grid][8] — a measurement aid, null in production.
  // 0 entry, 1 setup done, 2 producer past the dependency wait, 3 first stage ready, 4 last MMA commit,
  // 5 first accumulator ready (epilogue warp 4), 6 epilogue done (warp 4), 7 exit
  unsigned long long* trace;
  // fused all-gather of B (GATHER kernels only).  B occupies bytes [g_off, g_off + g_rows*g_row_bytes) of a
  // flat parameter unit that is split into equal shards of g_shard_bytes; shard r is at g_src.p[r] (a peer
  // mapping for the other ranks) and the local copy of the unit starts at g_dst.  Rows are N rows of a
  // K-major B or K rows of an MN-major B; chunk c = rows [64c, 64c+64), copied as g_pieces pieces.
  PeerTable g_src;
  uint8_t* g_dst;
  long long g_off, g_shard_bytes, g_row_bytes;
  int g_rows, g_chunks, g_pieces, g_world;
  unsigned* g_flags;  // [g_chunks] pieces arrived; zero between launches (the last CTA to exit resets them)
  unsigned* g_ctr;    // [2] piece claim counter, exited CTAs; zero between launches
  // decode consumer run by all CTAs after a grid-wide barrier (stream-K launches only; dec_fused.cuh)
  int consumer;
  unsigned* gbar;
  DecArgs dec;
  int group_m;  // M-tiles per raster group (tile_coords); 16 unless a pair launch picks another
};

constexpr int kGatherPiece = 16384;   // bytes per claimed piece
constexpr int kGatherMaxChunks = 8192;  // ready bits kept in shared memory by the producer

VLM_DEV void trace_mark(const GemmParams& p, int k) {
  if (p.trace) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    p.trace[blockIdx.x * 8 + k] = t;
  }
}

// Work item: one accumulation segment of one output tile.
struct Work {
  int tile, kb0, kb1, slot;
};

struct WorkIter {
  int kb_count, units_total;
  long long u, u_end, U;
  int t, grid;
  // pair: CTAs 2c and 2c+1 (one cluster) walk the same tiles, c = 0 .. gridDim.x/2 - 1
  VLM_DEV WorkIter(const GemmParams& p, int kbc, bool pair = false) : kb_count(kbc) {
    grid = gridDim.x >> (pair ? 1 : 0);
    units_total = p.tiles_m * p.tiles_n * p.splits;
    t = blockIdx.x >> (pair ? 1 : 0);
    U = static_cast<long long>(p.tiles_m) * p.tiles_n * kbc;
    u = (static_cast<long long>(blockIdx.x) * U) / grid;
    u_end = (static_cast<long long>(blockIdx.x + 1) * U) / grid;
  }
  VLM_DEV long long cta_of(long long x) const { return ((x + 1) * grid - 1) / U; }
  // number of CTAs whose unit range intersects `tile`
  VLM_DEV int slots_of(int tile) const {
    const long long first = static_cast<long long>(tile) * kb_count;
    return static_cast<int>(cta_of(first + kb_count - 1) - cta_of(first) + 1);
  }
  VLM_DEV bool next(const GemmParams& p, Work& w) {
    if (!p.streamk) {
      if (t >= units_total) return false;
      w.tile = t / p.splits;
      w.slot = t % p.splits;
      w.kb0 = w.slot * p.kb_per_split;
      w.kb1 = min(kb_count, w.kb0 + p.kb_per_split);
      t += grid;
      return true;
    }
    if (u >= u_end) return false;
    w.tile = static_cast<int>(u / kb_count);
    w.kb0 = static_cast<int>(u % kb_count);
    w.kb1 = static_cast<int>(min(static_cast<long long>(kb_count), w.kb0 + (u_end - u)));
    w.slot = static_cast<int>(blockIdx.x - cta_of(static_cast<long long>(w.tile) * kb_count));
    u += w.kb1 - w.kb0;
    return true;
  }
};

constexpr int kBM = 128;
constexpr int kBK = 64;

// PAIR: a 256 x BN tile on a CTA pair; each CTA stages 128 rows of A and BN/2 rows of B per k-block.
template <int BN, bool PAIR = false>
struct GemmCfg {
  static constexpr int BNC = PAIR ? BN / 2 : BN;  // B rows (N) staged by this CTA
  static constexpr int STAGES = PAIR ? (BN == 256 ? 6 : 8) : (BN == 256 ? 4 : 6);
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int B_BYTES = BNC * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  // per epilogue warp: a 32 x 16 fp32 staging tile (rows padded to 20 words) for coalesced partial stores
  static constexpr int EPI_STAGE_FLOATS = 32 * 20;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256 + 4 * EPI_STAGE_FLOATS * 4 + kGatherMaxChunks / 8;
};

// Tile t -> (tm, tn): groups of G M-tiles, walked M-fastest inside a group, so the CTAs of a wave share
// their B tiles (and G of A) in L2.  Stream-K consumers (streamk.cuh) assume G = 16.
VLM_DEV void tile_coords(int t, int tiles_m, int tiles_n, int& tm, int& tn, int G = 16) {
  const int group = G * tiles_n;
  const int gid = t / group;
  const int first = gid * G;
  const int gsz = min(tiles_m - first, G);
  const int r = t - gid * group;
  tm = first + r % gsz;
  tn = r / gsz;
}

VLM_DEV float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  return 0.5f * x * (1.f + tanhf(k0 * (x + k1 * x * x * x)));
}
VLM_DEV float gelu_erf(float x) { return 0.5f * x * (1.f + erff(x * 0.7071067811865476f)); }
VLM_DEV float silu(float x) { return x / (1.f + __expf(-x)); }

VLM_DEV void epilogue_chunk(const GemmParams& p, int row, int col, const uint32_t (&r)[16]) {
  float v[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]) * p.alpha;
  const int ncols = min(16, p.N - col);
  const bool full = ncols == 16;
  if (p.epi == EPI_SWIGLU_BWD) {
    // v = dL/d act for columns [col, col+16); aux row holds (gate, up) pairs at 2c, 2c+1.  d act is rounded to
    // bf16 first, like the unfused bf16 GEMM followed by the elementwise backward.
    const __nv_bfloat16* pre = p.aux + static_cast<long long>(row) * p.ld_aux + 2 * col;
    __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(p.D) + static_cast<long long>(row) * p.ldd + 2 * col;
    if (full) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 g4 = reinterpret_cast<const uint4*>(pre)[q];
        const uint32_t w[4] = {g4.x, g4.y, g4.z, g4.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 gu = unpack_bf16x2(w[j]);
          const float s = 1.f / (1.f + __expf(-gu.x));
          const float da = bf2f(f2bf(v[4 * q + j]));
          o[j] = pack_bf16x2(da * gu.y * s * (1.f + gu.x * (1.f - s)), da * gu.x * s);
        }
        reinterpret_cast<uint4*>(d)[q] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    } else {
      for (int i = 0; i < ncols; ++i) {
        const float g = bf2f(pre[2 * i]), u = bf2f(pre[2 * i + 1]);
        const float s = 1.f / (1.f + __expf(-g));
        const float da = bf2f(f2bf(v[i]));
        d[2 * i] = f2bf(da * u * s * (1.f + g * (1.f - s)));
        d[2 * i + 1] = f2bf(da * g * s);
      }
    }
    return;
  }
  if (p.epi == EPI_SWIGLU) {
    if (p.aux) {
      __nv_bfloat16* a = p.aux + static_cast<long long>(row) * p.ld_aux + col;
      if (full) {
        uint4 w0 = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                              pack_bf16x2(v[6], v[7]));
        uint4 w1 = make_uint4(pack_bf16x2(v[8], v[9]), pack_bf16x2(v[10], v[11]), pack_bf16x2(v[12], v[13]),
                              pack_bf16x2(v[14], v[15]));
        reinterpret_cast<uint4*>(a)[0] = w0;
        reinterpret_cast<uint4*>(a)[1] = w1;
      } else {
        for (int i = 0; i < ncols; ++i) a[i] = f2bf(v[i]);
      }
    }
    // gate/up are rounded to bf16 first, like an unfused bf16 GEMM followed by the activation
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float g = bf2f(f2bf(v[2 * j])), u = bf2f(f2bf(v[2 * j + 1]));
      o[j] = silu(g) * u;
    }
    __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(p.D) + static_cast<long long>(row) * p.ldd + col / 2;
    if (full) {
      reinterpret_cast<uint4*>(d)[0] =
          make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
    } else {
      for (int j = 0; j < ncols / 2; ++j) d[j] = f2bf(o[j]);
    }
    return;
  }
  if (p.bias) {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (i < ncols) v[i] += bf2f(p.bias[col + i]);
  }
  if (p.epi == EPI_GELU_TANH) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = gelu_tanh(v[i]);
  } else if (p.epi == EPI_GELU_ERF) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = gelu_erf(v[i]);
  }
  if (p.residual) {
    const __nv_bfloat16* rs = p.residual + static_cast<long long>(row) * p.ldr + col;
    if (full) {
      const uint4 a = reinterpret_cast<const uint4*>(rs)[0], b = reinterpret_cast<const uint4*>(rs)[1];
      const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float2 f = unpack_bf16x2(w[j]);
        v[2 * j] += f.x;
        v[2 * j + 1] += f.y;
      }
    } else {
      for (int i = 0; i < ncols; ++i) v[i] += bf2f(rs[i]);
    }
  }
  if (p.d_f32) {
    float* d = reinterpret_cast<float*>(p.D) + static_cast<long long>(row) * p.ldd + col;
    if (full) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float4 x = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        if (p.accumulate) {
          const float4 o = reinterpret_cast<const float4*>(d)[j];
          x.x += o.x;
          x.y += o.y;
          x.z += o.z;
          x.w += o.w;
        }
        reinterpret_cast<float4*>(d)[j] = x;
      }
    } else {
      for (int i = 0; i < ncols; ++i) d[i] = p.accumulate ? d[i] + v[i] : v[i];
    }
  } else {
    __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(p.D) + static_cast<long long>(row) * p.ldd + col;
    if (full) {
      reinterpret_cast<uint4*>(d)[0] =
          make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
      reinterpret_cast<uint4*>(d)[1] = make_uint4(pack_bf16x2(v[8], v[9]), pack_bf16x2(v[10], v[11]),
                                                  pack_bf16x2(v[12], v[13]), pack_bf16x2(v[14], v[15]));
    } else {
      for (int i = 0; i < ncols; ++i) d[i] = f2bf(v[i]);
    }
  }
}

VLM_DEV unsigned ld_acquire_gpu_u32(const unsigned* a) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}
VLM_DEV void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Producer side of the fused gather: wait until chunks [c0, c1) have all their pieces.  `ready` caches the
// chunks this CTA already saw complete.  The proxy fence orders the acquire before the TMA (async proxy)
// reads of the chunk.
VLM_DEV bool gather_wait(const GemmParams& p, uint32_t* ready, int c0, int c1, volatile int* abort_flag) {
  bool fresh = false;
  if (c0 < 0 || c1 > p.g_chunks) {  // never expected: chunk ranges come from in-range tiles
    *abort_flag = 1;
    atomicCAS(p.err, 0, kErrBadArgs);
    return false;
  }
  for (int c = c0; c < c1; ++c) {
    const uint32_t bit = 1u << (c & 31);
    if (ready[c >> 5] & bit) continue;
    if (ld_acquire_gpu_u32(p.g_flags + c) < static_cast<unsigned>(p.g_pieces)) {
      const long long t0 = clock64();
      while (ld_acquire_gpu_u32(p.g_flags + c) < static_cast<unsigned>(p.g_pieces)) {
        if (*abort_flag) return false;
        if (clock64() - t0 > kWaitCycles) {
          *abort_flag = 1;
          atomicCAS(p.err, 0, kErrTimeoutGather);
          return false;
        }
      }
    }
    ready[c >> 5] |= bit;
    fresh = true;
  }
  if (fresh) fence_proxy_async_global();
  return true;
}

// Copy warps of the fused gather: claim 16 KB pieces in chunk order until the queue is empty.  Nothing here
// waits on another CTA, so the copy makes progress whichever CTAs are resident.
VLM_DEV void gather_copy(const GemmParams& p, int lane) {
  constexpr int U = 16;  // 16-byte vectors in flight per lane
  const unsigned total = static_cast<unsigned>(p.g_chunks) * static_cast<unsigned>(p.g_pieces);
  const long long chunk_bytes = 64ll * p.g_row_bytes;
  const long long b_bytes = static_cast<long long>(p.g_rows) * p.g_row_bytes;
  const long long SB = p.g_shard_bytes;
  while (true) {
    unsigned idx = 0;
    if (lane == 0) idx = atomicAdd(p.g_ctr, 1u);
    idx = __shfl_sync(0xffffffffu, idx, 0);
    if (idx >= total) break;
    const int c = static_cast<int>(idx / p.g_pieces), j = static_cast<int>(idx % p.g_pieces);
    const long long b0 = c * chunk_bytes + static_cast<long long>(j) * kGatherPiece;
    const long long b1 = min(min(b0 + kGatherPiece, (c + 1) * chunk_bytes), b_bytes);
    if (b0 < b1) {
      const long long u0 = p.g_off + b0;
      const int o0 = static_cast<int>(u0 / SB), o1 = static_cast<int>((p.g_off + b1 - 1) / SB);
      for (long long x0 = b0; x0 < b1; x0 += 32ll * 16 * U) {
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const long long x = x0 + (u * 32 + lane) * 16ll;
          v[u] = make_uint4(0, 0, 0, 0);
          if (x < b1) {
            const long long ux = p.g_off + x;
            const int o = o0 == o1 ? o0 : static_cast<int>(ux / SB);
            const long long off = ux - o * SB;
            if (o >= 0 && o < p.g_world && off >= 0 && off + 16 <= SB) {
              v[u] = __ldcg(reinterpret_cast<const uint4*>(p.g_src.p[o] + off));
            } else {
              atomicCAS(p.err, 0, kErrBadArgs);  // never expected: the host checked the unit geometry
            }
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const long long x = x0 + (u * 32 + lane) * 16ll;
          if (x < b1 && p.g_off + x + 16 <= p.g_world * SB) __stcg(reinterpret_cast<uint4*>(p.g_dst + p.g_off + x), v[u]);
        }
      }
    }
    // publish the piece: generic stores -> async proxy (the consumer's TMA), then a release count
    fence_proxy_async_global();
    __threadfence();
    __syncwarp();
    if (lane == 0 && c < p.g_chunks)
      asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.g_flags + c) : "memory");
  }
}

// PAIR kernels run as clusters of 2 CTAs (cta_group::2): the leader (rank 0) issues the 128-row-per-CTA
// MMAs of a 256-row tile; both CTAs load their rows of A and their half of B (TMA completion counted on the
// leader's barrier), and both drain their own TMEM rows.
template <int BN, bool A_MN, bool B_MN, bool GATHER = false, bool PAIR = false>
__global__ void __launch_bounds__(GATHER ? 256 : 192, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmParams p) {
  using C = GemmCfg<BN, PAIR>;
  static_assert(!(PAIR && GATHER), "pair tiles do not gather");
  constexpr int TILE_M = PAIR ? 2 * kBM : kBM;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* epi_stage = reinterpret_cast<float*>(smem + C::STAGES * C::STAGE_BYTES + 256);
  uint32_t* gather_ready = reinterpret_cast<uint32_t*>(epi_stage + 4 * C::EPI_STAGE_FLOATS);
  int* last_cta = reinterpret_cast<int*>(tmem_holder + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb_count = (p.K + kBK - 1) / kBK;
  uint32_t rank = 0;
  if constexpr (PAIR) rank = cluster_ctarank();
  const bool leader = rank == 0;
  if (threadIdx.x == 0) trace_mark(p, 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], PAIR ? 8 : 4);  // the epilogue warps of both CTAs release an accumulator
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    if constexpr (GATHER) {
      for (int i = 0; i < (p.g_chunks + 31) / 32; ++i) gather_ready[i] = 0;
    }
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  // Programmatic dependent launch: the weight operand B (never written by earlier kernels of the step) of
  // the first STAGES k-blocks is requested right after the barriers exist — before the TMEM allocation
  // and the CTA barrier, and before waiting for the previous kernel.  Thread 0 is the TMA producer.
  int prefetched = 0;
  if (!PAIR && threadIdx.x == 0 && p.b_prefetch) {
    WorkIter it0(p, kb_count);
    Work w0;
    if (it0.next(p, w0)) {
      int tm0, tn0;
      tile_coords(w0.tile, p.tiles_m, p.tiles_n, tm0, tn0, p.group_m);
      prefetched = min(C::STAGES, w0.kb1 - w0.kb0);
      for (int i = 0; i < prefetched; ++i) {
        mbar_arrive_expect_tx(&full[i], C::STAGE_BYTES);
        uint8_t* b = sB + i * C::B_BYTES;
        const int k0 = (w0.kb0 + i) * kBK, n0 = tn0 * BN;
        if constexpr (!B_MN) {
          tma_load_2d(b, &tmB, &full[i], k0, n0);
        } else {
#pragma unroll
          for (int j = 0; j < BN / 64; ++j) tma_load_2d(b + j * 8192, &tmB, &full[i], n0 + 64 * j, k0);
        }
      }
    }
  }
  if (warp == 1) {
    if constexpr (PAIR) {  // the same warp of both CTAs allocates the pair's TMEM
      tmem_alloc_pair(tmem_holder, C::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_holder, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // the leader's barriers exist before the peer's copies signal them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  if (threadIdx.x == 0) trace_mark(p, 1);

  if (warp == 0) {
    if (lane == 0) {
      long long issued = 0;
      bool ok = true;
      int stage = 0;
      uint32_t phase = 0;
      // one 2-D load into this CTA's stage; PAIR: completion counted on the leader's full barrier
      auto ld = [&](uint8_t* dst, const CUtensorMap* map, int x, int y) {
        if constexpr (PAIR)
          tma_load_2d_pair(dst, map, mapa_shared(smem_u32(&full[stage]), 0), x, y);
        else
          tma_load_2d(dst, map, &full[stage], x, y);
      };
      auto load_b = [&](uint8_t* b, int k0, int n0) {
        if constexpr (!B_MN) {
          ld(b, &tmB, k0, n0);
        } else {
#pragma unroll
          for (int j = 0; j < C::BNC / 64; ++j) ld(b + j * 8192, &tmB, n0 + 64 * j, k0);
        }
      };
      WorkIter it(p, kb_count, PAIR);
      Work w;
      pdl_wait();
      trace_mark(p, 2);
      while (ok && it.next(p, w)) {
        int tm, tn;
        tile_coords(w.tile, p.tiles_m, p.tiles_n, tm, tn, p.group_m);
        const int m0 = tm * TILE_M + static_cast<int>(rank) * kBM, n0 = tn * BN + static_cast<int>(rank) * C::BNC;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          const bool pre = prefetched > 0;
          if (!pre && !mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          if constexpr (GATHER) {
            // K-major B: the tile's BN weight rows (chunks n0/64 ...); MN-major B: this k-block's 64 rows
            const int c0 = B_MN ? kb : n0 / 64;
            const int c1 = B_MN ? kb + 1 : min(p.g_chunks, (n0 + BN + 63) / 64);
            if ((B_MN || kb == w.kb0) && !gather_wait(p, gather_ready, c0, c1, abort_flag)) {
              ok = false;
              break;
            }
          }
          uint8_t* a = sA + stage * C::A_BYTES;
          uint8_t* b = sB + stage * C::B_BYTES;
          // PAIR: the leader expects the bytes of both CTAs on its barrier (the peer's may land first)
          if (!pre && leader) mbar_arrive_expect_tx(&full[stage], (PAIR ? 2 : 1) * C::STAGE_BYTES);
          const int k0 = kb * kBK;
          if constexpr (!A_MN) {
            ld(a, &tmA, k0, m0);
          } else {
            ld(a, &tmA, m0, k0);
            ld(a + 8192, &tmA, m0 + 64, k0);
          }
          if (!pre) load_b(b, k0, n0);
          if (pre) --prefetched;
          ++issued;
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && !PAIR) {
        // drain this thread's in-flight copies (at most STAGES) before the CTA exits
        for (long long i = issued - 1; i >= 0 && i >= issued - C::STAGES; --i) {
          volatile int no_abort = 0;
          mbar_wait(&full[i % C::STAGES], static_cast<uint32_t>((i / C::STAGES) & 1), &no_abort, nullptr, 0);
        }
      }
      if (!ok && PAIR) {
        // a pair's copies complete on the leader's barrier, which the peer cannot wait on: give this CTA's
        // own in-flight copies time to land before the teardown (error path only)
        for (int i = 0; i < 2000; ++i) __nanosleep(1000);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = idesc_bf16_f32(TILE_M, BN, A_MN, B_MN);
      bool ok = true;
      int stage = 0;
      uint32_t phase = 0;
      int lt = 0;
      WorkIter it(p, kb_count, PAIR);
      Work w;
      for (; ok && it.next(p, w); ++lt) {
        const int acc = lt & 1;
        const uint32_t use = static_cast<uint32_t>(lt >> 1);
        const bool freed = PAIR ? mbar_wait_cluster(&tempty[acc], (use & 1u) ^ 1u, abort_flag, p.err, kErrTimeoutMma)
                                : mbar_wait(&tempty[acc], (use & 1u) ^ 1u, abort_flag, p.err, kErrTimeoutMma);
        if (!freed) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        const int kb0 = w.kb0, kb1 = w.kb1;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          if (lt == 0 && kb == kb0) trace_mark(p, 3);
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = A_MN ? sdesc_sw128(a_addr + k * 2048, 8192, 1024) : sdesc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(b_addr + k * 2048, 8192, 1024) : sdesc_sw128(b_addr + k * 32, 16, 1024);
            if constexpr (PAIR)
              umma_f16_pair(d_tmem, ad, bd, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
            else
              umma_f16(d_tmem, ad, bd, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
          }
          if constexpr (PAIR)
            umma_commit_pair(&empty[stage]);  // frees the stage in both CTAs
          else
            umma_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if constexpr (PAIR)
          umma_commit_pair(&tfull[acc]);
        else
          umma_commit(&tfull[acc]);
        trace_mark(p, 4);
      }
      if (!ok) {
        if constexpr (PAIR)
          umma_commit_pair(drain);
        else
          umma_commit(drain);
        volatile int no_abort = 0;
        mbar_wait(drain, 0, &no_abort, nullptr, 0);
      }
    }
  } else if (GATHER && warp >= 6) {
    pdl_wait();  // the previous kernel may still read the buffer being filled
    gather_copy(p, lane);
  } else {
    pdl_wait();  // epilogue reads residual / writes outputs the previous kernel may still touch
    if (threadIdx.x == 64) pdl_trigger();  // only after the wait: dependents never overlap our predecessor
    const int q = warp & 3;  // TMEM lanes [32q, 32q+32) are the ones this warp may read
    const int row_in_tile = q * 32 + lane;
    int lt = 0;
    WorkIter it(p, kb_count, PAIR);
    Work w;
    for (; it.next(p, w); ++lt) {
      const int acc = lt & 1;
      const uint32_t use = static_cast<uint32_t>(lt >> 1);
      if (!mbar_wait(&tfull[acc], use & 1u, abort_flag, p.err, kErrTimeoutEpilogue)) break;
      if (threadIdx.x == 128 && lt == 0) trace_mark(p, 5);
      tc_fence_after();
      int tm, tn;
      tile_coords(w.tile, p.tiles_m, p.tiles_n, tm, tn, p.group_m);
      const int m_base = tm * TILE_M + static_cast<int>(rank) * kBM;  // this CTA's 128 rows of the tile
      const int row = m_base + row_in_tile;
      const int n0 = tn * BN;
      const uint32_t tbase = tmem_base + static_cast<uint32_t>(acc * BN) + (static_cast<uint32_t>(q * 32) << 16);
      if (m_base + q * 32 >= p.M) {
        // every row of this warp's TMEM lanes is past M (decode-shaped M): nothing to load or store
      } else if (p.streamk) {
        // Each lane holds one row's 16 columns after tcgen05.ld; storing that directly makes every warp
        // store touch 32 rows.  Stage the 32 x 16 block in shared memory and store it transposed: lane
        // (r4, c) writes 16 bytes of row 8*i + r4, so one store instruction covers 8 rows x 64 bytes.
        float* stg = epi_stage + (warp - 2) * C::EPI_STAGE_FLOATS;
        const int row_base = m_base + q * 32;
        const int sr = lane >> 2, sc = (lane & 3) * 4;
#pragma unroll 1
        for (int c4 = 0; c4 < BN; c4 += 128) {
          uint32_t rr[8][16];
#pragma unroll
          for (int j = 0; j < 8; ++j) tmem_ld16(tbase + c4 + 16 * j, rr[j]);
          tmem_ld_wait();  // one round trip per 128 columns
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int col0 = n0 + c4 + 16 * j;
            if (col0 >= p.N) continue;  // warp-uniform
#pragma unroll
            for (int i = 0; i < 4; ++i)
              reinterpret_cast<float4*>(stg + lane * 20)[i] =
                  make_float4(__uint_as_float(rr[j][4 * i]), __uint_as_float(rr[j][4 * i + 1]),
                              __uint_as_float(rr[j][4 * i + 2]), __uint_as_float(rr[j][4 * i + 3]));
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int r = 8 * i + sr;
              const int grow = row_base + r;
              if (grow < p.M) {
                const float4 v4 = *reinterpret_cast<const float4*>(stg + r * 20 + sc);
                float* dst = p.ws + (static_cast<int64_t>(w.slot) * p.M + grow) * p.N + col0 + sc;
                if (col0 + sc + 4 <= p.N) {
                  *reinterpret_cast<float4*>(dst) = v4;
                } else {
                  const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
                  for (int e = 0; e < 4 && col0 + sc + e < p.N; ++e) dst[e] = vv[e];
                }
              }
            }
            __syncwarp();
          }
        }
      } else if (p.epi == EPI_VOCAB_STATS) {
        // online (max, sum exp, sum exp*z) of this row over the tile's columns; never stores logits
        float mx = -INFINITY, se = 0.f, sz = 0.f, zt = __int_as_float(0x7fc00000);
        const int64_t tgt = row < p.M ? p.targets[row] : -1;
#pragma unroll 1
        for (int c4 = 0; c4 < BN; c4 += 64) {
          uint32_t rr[4][16];
#pragma unroll
          for (int j = 0; j < 4; ++j) tmem_ld16(tbase + c4 + 16 * j, rr[j]);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 4; ++j) {
          const uint32_t (&r)[16] = rr[j];
          const int col0 = n0 + c4 + 16 * j;
          const int nv = min(16, p.N - col0);
          if (nv <= 0) continue;
          float cm = -INFINITY;
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (i < nv) cm = fmaxf(cm, __uint_as_float(r[i]) * p.alpha);
          if (cm > mx) {
            const float sc = __expf(mx - cm);
            se *= sc;
            sz *= sc;
            mx = cm;
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if (i < nv) {
              const float z = __uint_as_float(r[i]) * p.alpha;
              const float e = __expf(z - mx);
              se += e;
              sz += e * z;
            }
          }
          if (tgt >= col0 && tgt < col0 + nv) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (col0 + i == tgt) zt = __uint_as_float(r[i]) * p.alpha;
          }
          }
        }
        if (row < p.M) {
          reinterpret_cast<float4*>(p.part)[static_cast<int64_t>(row) * p.tiles_n + tn] = make_float4(mx, se, sz, zt);
        }
      } else if (p.epi == EPI_TOPK) {
        // this row's topk largest logits of the tile (value desc, index asc), found by topk selection passes
        // over the accumulator (each pass re-reads TMEM and takes the best entry after the previous pick);
        // scalar state only, no per-lane divergence, and the logits are never stored
        const int kk = p.topk;
        const int64_t base = (static_cast<int64_t>(row) * p.tiles_n + tn) * kk;
        float pv = INFINITY;
        int pi = -1;
#pragma unroll 1
        for (int r = 0; r < kk; ++r) {
          float bv = -INFINITY;
          int bi = 0x7fffffff;
#pragma unroll 1
          for (int c4 = 0; c4 < BN; c4 += 64) {
            uint32_t rr[4][16];
#pragma unroll
            for (int j = 0; j < 4; ++j) tmem_ld16(tbase + c4 + 16 * j, rr[j]);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int col0 = n0 + c4 + 16 * j;
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const float z = __uint_as_float(rr[j][i]) * p.alpha;
                const int zi = col0 + i;
                const bool after = z < pv || (z == pv && zi > pi);  // not picked yet
                const bool better = z > bv || (z == bv && zi < bi);
                if (zi < p.N && after && better) {
                  bv = z;
                  bi = zi;
                }
              }
            }
          }
          if (row < p.M) {
            p.part[base + r] = bv;
            p.cand_i[base + r] = bi;
          }
          pv = bv;
          pi = bi;
        }
      } else if (p.epi == EPI_VOCAB_GRAD) {
        // dlogits = g_lp * (onehot - p) - g_ent * p * (log p + H), p = exp(z - lse)
        float lse = 0.f, ent = 0.f, glp = 0.f, gent = 0.f;
        int64_t tgt = -1;
        if (row < p.M) {
          lse = p.row_lse[row];
          ent = p.row_ent[row];
          glp = p.g_lp[row];
          gent = p.g_ent[row];
          tgt = p.targets[row];
        }
#pragma unroll 1
        for (int c4 = 0; c4 < BN; c4 += 64) {
          uint32_t rr[4][16];
#pragma unroll
          for (int j = 0; j < 4; ++j) tmem_ld16(tbase + c4 + 16 * j, rr[j]);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 4; ++j) {
          const uint32_t (&r)[16] = rr[j];
          const int col0 = n0 + c4 + 16 * j;
          if (row >= p.M || col0 >= p.N) continue;
          float v[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float lp = __uint_as_float(r[i]) * p.alpha - lse;
            const float pr = __expf(lp);
            v[i] = -glp * pr - gent * pr * (lp + ent) + (col0 + i == tgt ? glp : 0.f);
          }
          __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(p.D) + static_cast<long long>(row) * p.ldd + col0;
          if (col0 + 16 <= p.N) {
            reinterpret_cast<uint4*>(d)[0] = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                                        pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
            reinterpret_cast<uint4*>(d)[1] = make_uint4(pack_bf16x2(v[8], v[9]), pack_bf16x2(v[10], v[11]),
                                                        pack_bf16x2(v[12], v[13]), pack_bf16x2(v[14], v[15]));
          } else {
            for (int i = 0; i < p.N - col0; ++i) d[i] = f2bf(v[i]);
          }
          }
        }
      } else {
#pragma unroll 1
        for (int c4 = 0; c4 < BN; c4 += 64) {
          uint32_t rr[4][16];
#pragma unroll
          for (int j = 0; j < 4; ++j) tmem_ld16(tbase + c4 + 16 * j, rr[j]);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (row < p.M && n0 + c4 + 16 * j < p.N) epilogue_chunk(p, row, n0 + c4 + 16 * j, rr[j]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR)
          mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));  // the leader's MMA waits on both CTAs
        else
          mbar_arrive(&tempty[acc]);
      }
      if (threadIdx.x == 128) trace_mark(p, 6);
    }
  }

  tc_fence_before();
  __syncthreads();
  // PAIR: neither CTA frees TMEM or leaves while the pair's MMAs, remote arrivals or copies may touch it
  if constexpr (PAIR) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    else
      tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if constexpr (GATHER) {
    // every role of this CTA is done with the gather state; the last CTA out zeroes it for the next launch
    if (threadIdx.x == 0) {
      __threadfence();
      *last_cta = atomicAdd(p.g_ctr + 1, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (*last_cta) {
      __threadfence();
      for (int c = threadIdx.x; c < p.g_chunks; c += blockDim.x) p.g_flags[c] = 0;
      if (threadIdx.x == 0) {
        p.g_ctr[0] = 0;
        p.g_ctr[1] = 0;
      }
    }
  }
  if constexpr (!A_MN && !B_MN && !GATHER) {
    if (p.consumer != DEC_NONE && dec_grid_sync(p.gbar, p.err, last_cta)) {
      const SkMeta m{p.M, p.N, p.tiles_m, p.tiles_n, kb_count, p.sk_grid, kBM, BN};
      if (p.consumer == DEC_QKV) {
        if (p.dec.head_dim == 128)
          dec_qkv_part<128>(p.ws, m, p.dec);
        else if (p.dec.head_dim == 64)
          dec_qkv_part<64>(p.ws, m, p.dec);
        else
          dec_qkv_part<32>(p.ws, m, p.dec);
      } else if (p.consumer == DEC_RESNORM) {
        dec_resnorm_part<4>(p.ws, m, p.dec, epi_stage);
      } else {
        dec_swiglu_part(p.ws, m, p.dec);
      }
    }
  }
  if (threadIdx.x == 0) trace_mark(p, 7);
}

// Generic consumer of stream-K partials: sums the slots of 16 columns and applies the GEMM epilogue.
__global__ void sk_reduce_kernel(GemmParams p, SkMeta m) {
  pdl_wait();
  const int chunks = (p.N + 15) / 16;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(p.M) * chunks) return;
  const int row = static_cast<int>(idx / chunks), col = static_cast<int>(idx % chunks) * 16;
  float a[8], b[8];
  sk_sum8(p.ws, m, row, col, a);
  if (col + 8 < p.N) {
    sk_sum8(p.ws, m, row, col + 8, b);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) b[i] = 0.f;
  }
  uint32_t r[16];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    r[i] = __float_as_uint(a[i]);
    r[8 + i] = __float_as_uint(b[i]);
  }
  epilogue_chunk(p, row, col, r);
}

// ------------------------------------------------------------------ host side
// Set while the weights are read-only (the decode loop): GEMMs may then stream B before the wait on
// their predecessor kernel.
static thread_local bool g_static_weights = false;
// Set only inside gemm_partials_traced: the next launch records per-CTA phase timestamps here.
static thread_local unsigned long long* g_trace = nullptr;
void set_static_weights(bool on) { g_static_weights = on; }

// Cluster-of-2 launch of a PAIR kernel (grid = 2 x pairs) with programmatic serialization.
template <int BN, bool A_MN, bool B_MN>
static void launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int pairs, cudaStream_t st) {
  auto kern = gemm_tcgen05_kernel<BN, A_MN, B_MN, false, true>;
  static bool configured = false;
  if (!configured) {
    VLM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<BN, true>::SMEM));
    VLM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = GemmCfg<BN, true>::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  unsigned n = 1;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  VLM_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, p));
  note_launch();
}

// How many 2-CTA clusters of the pair kernel can be resident at once (cached per tile width).
template <int BN>
static int max_pairs(int device) {
  static int cached[64] = {0};
  if (!cached[device]) {
    auto kern = gemm_tcgen05_kernel<BN, false, false, false, true>;
    VLM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<BN, true>::SMEM));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 148);
    cfg.blockDim = dim3(192);
    cfg.dynamicSmemBytes = GemmCfg<BN, true>::SMEM;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    VLM_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
    cached[device] = std::max(1, n);
  }
  return cached[device];
}

// M-tiles per raster group of pair launches (VLMRL_GEMM_GROUP overrides, for measurements).
static int pair_group() {
  static const int g = [] {
    const char* e = std::getenv("VLMRL_GEMM_GROUP");
    return e ? std::max(1, std::atoi(e)) : 16;
  }();
  return g;
}

static bool pair_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("VLMRL_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <int BN, bool A_MN, bool B_MN, bool GATHER = false>
static void launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int grid, cudaStream_t st) {
  auto kern = gemm_tcgen05_kernel<BN, A_MN, B_MN, GATHER>;
  static bool configured = false;
  if (!configured) {
    VLM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<BN>::SMEM));
    configured = true;
  }
  // a fused decode consumer waits at a grid-wide barrier: cooperative launch keeps every CTA resident
  // (VLMRL_DECODE_COOP=0 drops the attribute, for timing only: grid <= #SMs at one CTA per SM)
  static const bool coop = [] {
    const char* e = std::getenv("VLMRL_DECODE_COOP");
    return !(e && e[0] == '0');
  }();
  launch_ex(p.consumer != DEC_NONE && coop, kern, dim3(grid), dim3(GATHER ? 256 : 192), GemmCfg<BN>::SMEM, st, ta, tb,
            p);
}

static void check_operand(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, name, " must be a CUDA bf16 tensor");
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, name, " must be 2-D with a contiguous inner dimension");
  TORCH_CHECK(t.stride(0) % 8 == 0 || t.size(0) == 1, name, " leading stride must be a multiple of 8 elements");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name, " must be 16-byte aligned");
}

void gemm_ex(at::Tensor A, at::Tensor B, at::Tensor D, at::Tensor bias, at::Tensor residual, at::Tensor aux,
             bool a_kmajor, bool b_kmajor, double alpha, int64_t epi, bool accumulate, const VocabArgs* vocab,
             int force_bn, at::Tensor* partials_out, SkMeta* meta_out, const GatherArgs* gather, const DecFuse* fuse) {
  check_operand(A, "A");
  check_operand(B, "B");
  const c10::cuda::CUDAGuard guard(A.device());
  const int64_t M = a_kmajor ? A.size(0) : A.size(1);
  const int64_t K = a_kmajor ? A.size(1) : A.size(0);
  const int64_t N = b_kmajor ? B.size(0) : B.size(1);
  const int64_t Kb = b_kmajor ? B.size(1) : B.size(0);
  TORCH_CHECK(K == Kb, "gemm: K mismatch ", K, " vs ", Kb);
  TORCH_CHECK(K > 0 && M > 0 && N > 0, "gemm: empty problem");
  TORCH_CHECK(N % 8 == 0, "gemm: N must be a multiple of 8");
  const bool want_partials = partials_out != nullptr;
  const bool is_stats = epi == EPI_VOCAB_STATS || epi == EPI_TOPK || want_partials;
  TORCH_CHECK(is_stats || (D.is_cuda() && D.dim() == 2 && D.stride(1) == 1), "gemm: bad output");
  TORCH_CHECK((epi != EPI_VOCAB_STATS && epi != EPI_VOCAB_GRAD && epi != EPI_TOPK) || vocab != nullptr,
              "gemm: vocab epilogue needs row data");
  TORCH_CHECK(epi != EPI_TOPK || (vocab->topk >= 1 && vocab->topk <= kTopkMax && vocab->cand_i && vocab->part),
              "gemm: top-k epilogue needs 1..", kTopkMax, " candidates per tile and candidate buffers");
  const bool d_f32 = !is_stats && D.scalar_type() == at::kFloat;
  if (!is_stats) {
    TORCH_CHECK(d_f32 || D.scalar_type() == at::kBFloat16, "gemm: output must be bf16 or fp32");
    TORCH_CHECK(!accumulate || d_f32, "gemm: accumulate needs an fp32 output");
    TORCH_CHECK(D.size(0) == M && D.size(1) == (epi == EPI_SWIGLU ? N / 2 : epi == EPI_SWIGLU_BWD ? 2 * N : N),
                "gemm: output shape mismatch");
    TORCH_CHECK(epi != EPI_SWIGLU_BWD || (aux.defined() && D.scalar_type() == at::kBFloat16 && !accumulate),
                "gemm: the SwiGLU-backward epilogue needs the forward's (gate, up) as aux and a bf16 output");
    TORCH_CHECK(D.stride(0) % 8 == 0, "gemm: output leading stride must be a multiple of 8");
  }

  GemmParams p{};
  p.group_m = 16;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.D = is_stats ? nullptr : D.data_ptr();
  p.ldd = is_stats ? 0 : D.stride(0);
  if (vocab) {
    p.targets = vocab->targets;
    p.row_lse = vocab->lse;
    p.row_ent = vocab->ent;
    p.g_lp = vocab->g_lp;
    p.g_ent = vocab->g_ent;
    p.part = vocab->part;
    p.cand_i = vocab->cand_i;
    p.topk = vocab->topk;
  }
  p.d_f32 = d_f32;
  p.alpha = static_cast<float>(alpha);
  p.epi = static_cast<int>(epi);
  p.accumulate = accumulate;
  p.err = err_word(A.device().index());
  p.trace = g_trace;
  // B is prefetched ahead of the dependency wait only when it is a K-major weight: the forward and
  // decode GEMMs.  Backward GEMMs (MN-major operands) read activation gradients as B.
  p.b_prefetch = (g_static_weights && b_kmajor && !accumulate && epi != EPI_VOCAB_GRAD && !gather) ? 1 : 0;
  if (gather) {
    const int W = static_cast<int>(gather->srcs.size());
    TORCH_CHECK(W >= 1 && W <= kMaxRanks, "gemm_gather: 1..", kMaxRanks, " shards");
    TORCH_CHECK(B.is_contiguous(), "gemm_gather: B must be a contiguous view of the unit");
    const int64_t rows = B.size(0), row_bytes = B.size(1) * 2;
    const int64_t off = reinterpret_cast<int64_t>(B.data_ptr()) - gather->dst_base;
    TORCH_CHECK(off >= 0 && off % 16 == 0 && off + rows * row_bytes <= W * gather->shard_bytes,
                "gemm_gather: B is not inside the unit");
    TORCH_CHECK(gather->shard_bytes % 16 == 0 && gather->dst_base % 16 == 0, "gemm_gather: 16-byte alignment");
    const int64_t chunks = (rows + 63) / 64;
    TORCH_CHECK(chunks <= kGatherMaxChunks, "gemm_gather: more than ", kGatherMaxChunks, " chunks");
    TORCH_CHECK(gather->flags.is_cuda() && gather->flags.scalar_type() == at::kInt && gather->flags.numel() >= chunks &&
                    gather->ctr.is_cuda() && gather->ctr.scalar_type() == at::kInt && gather->ctr.numel() >= 2,
                "gemm_gather: flags int32 [>= chunks] and ctr int32 [2] on the device");
    TORCH_CHECK(!partials_out && epi != EPI_VOCAB_STATS, "gemm_gather: not with partial-sum outputs");
    p.g_src = make_peer_table(gather->srcs);
    p.g_dst = reinterpret_cast<uint8_t*>(gather->dst_base);
    p.g_off = off;
    p.g_shard_bytes = gather->shard_bytes;
    p.g_row_bytes = row_bytes;
    p.g_rows = static_cast<int>(rows);
    p.g_chunks = static_cast<int>(chunks);
    p.g_pieces = static_cast<int>((64 * row_bytes + kGatherPiece - 1) / kGatherPiece);
    p.g_world = W;
    p.g_flags = reinterpret_cast<unsigned*>(gather->flags.data_ptr());
    p.g_ctr = reinterpret_cast<unsigned*>(gather->ctr.data_ptr());
  }
  if (bias.defined() && bias.numel()) {
    TORCH_CHECK(bias.scalar_type() == at::kBFloat16 && bias.is_contiguous() && bias.numel() == N, "gemm: bad bias");
    p.bias = reinterpret_cast<const __nv_bfloat16*>(bias.data_ptr());
  }
  if (residual.defined() && residual.numel()) {
    TORCH_CHECK(residual.scalar_type() == at::kBFloat16 && residual.stride(1) == 1 && residual.size(0) == M &&
                    residual.size(1) == N && residual.stride(0) % 8 == 0,
                "gemm: bad residual");
    p.residual = reinterpret_cast<const __nv_bfloat16*>(residual.data_ptr());
    p.ldr = residual.stride(0);
  }
  if (aux.defined() && aux.numel()) {
    TORCH_CHECK(aux.scalar_type() == at::kBFloat16 && aux.stride(1) == 1 && aux.size(0) == M &&
                    aux.size(1) == (epi == EPI_SWIGLU_BWD ? 2 * N : N) && aux.stride(0) % 8 == 0,
                "gemm: bad aux");
    p.aux = reinterpret_cast<__nv_bfloat16*>(aux.data_ptr());
    p.ld_aux = aux.stride(0);
  }

  // Training-sized GEMMs run on CTA pairs (256-row tiles, half of B per SM): fewer operand bytes per FLOP
  // through L2 than single-CTA 128-row tiles.  Decode (stream-K), gather, vocab and fused-consumer GEMMs
  // keep the single-CTA kernel.  VLMRL_GEMM_PAIR=0 turns pairs off.
  const bool use_pair = pair_enabled() && !gather && !fuse && !want_partials && epi != EPI_VOCAB_STATS && epi != EPI_TOPK &&
                        epi != EPI_VOCAB_GRAD && force_bn == 0 && (a_kmajor || !b_kmajor) && M >= 4 * kBM;
  if (use_pair) {
    // Always 256-wide: 128-wide pair tiles (64 B rows per CTA) measured at about 0.5 of the bf16 peak on
    // every training shape, 256-wide at 0.70-0.85, even where 128 would fill the last wave better.
    const int dev = A.device().index();
    const int64_t tm2 = (M + 2 * kBM - 1) / (2 * kBM);
    const int bn = 256;
    p.tiles_m = static_cast<int>(tm2);
    p.tiles_n = static_cast<int>((N + bn - 1) / bn);
    p.bn = bn;
    p.splits = 1;
    p.kb_per_split = static_cast<int>((K + kBK - 1) / kBK);
    p.streamk = 0;
    p.b_prefetch = 0;
    p.group_m = pair_group();
    const int64_t tiles2 = static_cast<int64_t>(p.tiles_m) * p.tiles_n;
    const int pairs = static_cast<int>(std::min<int64_t>(tiles2, max_pairs<256>(dev)));
    CUtensorMap ta, tb;
    if (a_kmajor)
      ta = make_tmap_2d_bf16(A.data_ptr(), K, M, A.stride(0), 64, 128);
    else
      ta = make_tmap_2d_bf16(A.data_ptr(), M, K, A.stride(0), 64, 64);
    if (b_kmajor)
      tb = make_tmap_2d_bf16(B.data_ptr(), K, N, B.stride(0), 64, bn / 2);
    else
      tb = make_tmap_2d_bf16(B.data_ptr(), N, K, B.stride(0), 64, 64);
    cudaStream_t st = at::cuda::getCurrentCUDAStream();
    if (a_kmajor && b_kmajor)
      launch_pair<256, false, false>(ta, tb, p, pairs, st);
    else if (a_kmajor)
      launch_pair<256, false, true>(ta, tb, p, pairs, st);
    else
      launch_pair<256, true, true>(ta, tb, p, pairs, st);
    return;
  }

  const int sms = num_sms(A.device().index());
  const int64_t tm_count = (M + kBM - 1) / kBM;
  // pick the tile width with the better wave efficiency (ties -> 256, the more efficient tile)
  auto wave_eff = [&](int bn) {
    const double t = static_cast<double>(tm_count * ((N + bn - 1) / bn));
    return t / (std::ceil(t / sms) * sms);
  };
  int BN = force_bn;
  if (!BN) BN = (M <= kBM || wave_eff(128) > wave_eff(256) + 0.1) ? 128 : 256;
  p.tiles_m = static_cast<int>(tm_count);
  p.tiles_n = static_cast<int>((N + BN - 1) / BN);
  const int64_t tiles = static_cast<int64_t>(p.tiles_m) * p.tiles_n;
  const int kb_count = static_cast<int>((K + kBK - 1) / kBK);
  // split-K for skinny problems that would leave most SMs idle
  int splits = 1;
  at::Tensor ws;
  const bool splittable = epi <= EPI_GELU_ERF && !accumulate;
  p.bn = BN;
  p.kb_per_split = kb_count;
  int grid = static_cast<int>(std::min<int64_t>(tiles, sms));
  // Skinny problems (decode, M <= 2 tiles): stream-K over (tile, k-block) units so every SM gets the
  // same amount of weight streaming; partial sums go to a [slots, M, N] fp32 workspace.
  const int64_t units = tiles * kb_count;
  if (fuse) {
    TORCH_CHECK(want_partials && !gather, "fused decode consumer: stream-K partials only");
    p.consumer = fuse->consumer;
    p.dec = fuse->args;
    p.gbar = grid_barrier_words(A.device().index());
  }
  if (want_partials || (splittable && p.tiles_m <= 2 && tiles < 4 * sms && units >= 2 * sms)) {
    TORCH_CHECK(!want_partials || (a_kmajor && b_kmajor && alpha == 1.0), "gemm partials: K-major operands only");
    p.streamk = 1;
    grid = static_cast<int>(std::min<int64_t>(sms, units));
    const int64_t per_cta = std::max<int64_t>(1, units / grid);
    const int64_t slots = std::min<int64_t>((kb_count + per_cta - 1) / per_cta + 1, grid);
    ws = at::empty({slots, M, N}, A.options().dtype(at::kFloat));
    p.ws = ws.data_ptr<float>();
    p.sk_grid = grid;
  }
  p.splits = splits;

  // tensor maps: inner dimension first
  CUtensorMap ta, tb;
  if (a_kmajor)
    ta = make_tmap_2d_bf16(A.data_ptr(), K, M, A.stride(0), 64, 128);
  else
    ta = make_tmap_2d_bf16(A.data_ptr(), M, K, A.stride(0), 64, 64);
  if (b_kmajor)
    tb = make_tmap_2d_bf16(B.data_ptr(), K, N, B.stride(0), 64, BN);
  else
    tb = make_tmap_2d_bf16(B.data_ptr(), N, K, B.stride(0), 64, 64);

  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (gather) {
    TORCH_CHECK(a_kmajor, "gemm_gather: K-major A only");
    if (b_kmajor)
      BN == 256 ? launch<256, false, false, true>(ta, tb, p, grid, st) : launch<128, false, false, true>(ta, tb, p, grid, st);
    else
      BN == 256 ? launch<256, false, true, true>(ta, tb, p, grid, st) : launch<128, false, true, true>(ta, tb, p, grid, st);
  } else if (a_kmajor && b_kmajor) {
    BN == 256 ? launch<256, false, false>(ta, tb, p, grid, st) : launch<128, false, false>(ta, tb, p, grid, st);
  } else if (a_kmajor && !b_kmajor) {
    BN == 256 ? launch<256, false, true>(ta, tb, p, grid, st) : launch<128, false, true>(ta, tb, p, grid, st);
  } else if (!a_kmajor && !b_kmajor) {
    BN == 256 ? launch<256, true, true>(ta, tb, p, grid, st) : launch<128, true, true>(ta, tb, p, grid, st);
  } else {
    TORCH_CHECK(false, "gemm: MN-major A with K-major B is not instantiated");
  }
  if (p.streamk) {
    SkMeta m{p.M, p.N, p.tiles_m, p.tiles_n, kb_count, grid, kBM, BN};
    if (want_partials) {
      *partials_out = ws;
      *meta_out = m;
    } else {
      const int64_t threads = M * ((N + 15) / 16);
      launch_pdl(sk_reduce_kernel, dim3(static_cast<int>((threads + 127) / 128)), dim3(128), 0, st, p, m);
    }
  }
}

void gemm(at::Tensor A, at::Tensor B, at::Tensor D, at::Tensor bias, at::Tensor residual, at::Tensor aux, bool a_kmajor,
          bool b_kmajor, double alpha, int64_t epi, bool accumulate) {
  TORCH_CHECK((epi >= EPI_STORE && epi <= EPI_GELU_ERF) || epi == EPI_SWIGLU_BWD, "gemm: epilogue code ", epi,
              " is internal");
  gemm_ex(A, B, D, bias, residual, aux, a_kmajor, b_kmajor, alpha, epi, accumulate, nullptr, 0, nullptr, nullptr);
}

void gemm_gather(at::Tensor A, at::Tensor B, at::Tensor D, at::Tensor bias, at::Tensor residual, at::Tensor aux,
                 bool a_kmajor, bool b_kmajor, double alpha, int64_t epi, bool accumulate, std::vector<int64_t> srcs,
                 int64_t dst_base, int64_t shard_bytes, at::Tensor flags, at::Tensor ctr) {
  TORCH_CHECK((epi >= EPI_STORE && epi <= EPI_GELU_ERF) || epi == EPI_SWIGLU_BWD, "gemm_gather: epilogue code ", epi,
              " is internal");
  GatherArgs g{std::move(srcs), dst_base, shard_bytes, flags, ctr};
  gemm_ex(A, B, D, bias, residual, aux, a_kmajor, b_kmajor, alpha, epi, accumulate, nullptr, 0, nullptr, nullptr, &g);
}

// Ranges of a sharded unit copied by a grid-stride loop of 16-byte vectors (ranges are 16-byte aligned).
struct UnitRanges {
  long long start[8], end[8];
  int n;
};

__global__ void unit_gather_kernel(PeerTable src, uint8_t* dst, long long SB, UnitRanges r) {
  pdl_wait();
  const long long tid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (int i = 0; i < r.n; ++i) {
    for (long long x = r.start[i] + tid * 16; x < r.end[i]; x += stride * 16) {
      const int o = static_cast<int>(x / SB);
      __stcg(reinterpret_cast<uint4*>(dst + x),
             __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(src.p[o]) + (x - o * SB))));
    }
  }
}

void unit_gather(std::vector<int64_t> srcs, int64_t dst_base, int64_t shard_bytes, std::vector<int64_t> starts,
                 std::vector<int64_t> ends) {
  TORCH_CHECK(starts.size() == ends.size() && !starts.empty() && starts.size() <= 8, "unit_gather: 1..8 ranges");
  TORCH_CHECK(shard_bytes % 16 == 0 && dst_base % 16 == 0, "unit_gather: 16-byte alignment");
  UnitRanges r{};
  r.n = static_cast<int>(starts.size());
  long long total = 0;
  for (int i = 0; i < r.n; ++i) {
    TORCH_CHECK(starts[i] % 16 == 0 && ends[i] % 16 == 0 && starts[i] <= ends[i] &&
                    ends[i] <= shard_bytes * static_cast<int64_t>(srcs.size()),
                "unit_gather: ranges must be 16-byte aligned and inside the unit");
    r.start[i] = starts[i];
    r.end[i] = ends[i];
    total = std::max<long long>(total, ends[i] - starts[i]);
  }
  if (total == 0) return;
  const int threads = 256;
  const int grid = static_cast<int>(std::min<long long>((total / 16 + threads - 1) / threads, 4 * 148));
  launch_pdl(unit_gather_kernel, dim3(grid), dim3(threads), 0, at::cuda::getCurrentCUDAStream(), make_peer_table(srcs),
             reinterpret_cast<uint8_t*>(dst_base), static_cast<long long>(shard_bytes), r);
}

// ------------------------------------------------------------------ decode GEMMs with fused consumers
static const bf16_t* bf16_ptr_or_null(const at::Tensor& t) {
  return t.defined() && t.numel() ? reinterpret_cast<const bf16_t*>(t.data_ptr()) : nullptr;
}

static void dec_gemm_run(const at::Tensor& x, const at::Tensor& w, DecFuse& f) {
  at::Tensor ws;
  SkMeta m{};
  gemm_ex(x, w, at::Tensor(), at::Tensor(), at::Tensor(), at::Tensor(), true, true, 1.0, EPI_STORE, false, nullptr, 0,
          &ws, &m, nullptr, &f);
}

at::Tensor dec_gemm_qkv(at::Tensor x, at::Tensor w, at::Tensor bias, at::Tensor qw, at::Tensor kw, at::Tensor lengths,
                        at::Tensor delta, at::Tensor inv_freq, at::Tensor kc, at::Tensor vc, int64_t nq, int64_t nkv,
                        double eps) {
  const int D = static_cast<int>(kc.size(-1));
  TORCH_CHECK(D == 128 || D == 64 || D == 32, "dec_gemm_qkv: head_dim 32, 64 or 128");
  TORCH_CHECK(w.size(0) == (nq + 2 * nkv) * D, "dec_gemm_qkv: width mismatch");
  TORCH_CHECK(lengths.scalar_type() == at::kInt && delta.scalar_type() == at::kLong, "dec_gemm_qkv: int32 lengths, int64 deltas");
  TORCH_CHECK(kc.is_contiguous() && vc.is_contiguous(), "dec_gemm_qkv: contiguous cache layer");
  const c10::cuda::CUDAGuard g(x.device());
  at::Tensor q = at::empty({x.size(0), nq, D}, kc.options());
  DecFuse f{};
  f.consumer = DEC_QKV;
  f.args.bias = bf16_ptr_or_null(bias);
  f.args.qw = bf16_ptr_or_null(qw);
  f.args.kw = bf16_ptr_or_null(kw);
  f.args.lengths = lengths.data_ptr<int>();
  f.args.delta = delta.data_ptr<int64_t>();
  f.args.inv_freq = inv_freq.data_ptr<float>();
  f.args.q = reinterpret_cast<bf16_t*>(q.data_ptr());
  f.args.kc = reinterpret_cast<bf16_t*>(kc.data_ptr());
  f.args.vc = reinterpret_cast<bf16_t*>(vc.data_ptr());
  f.args.nq = static_cast<int>(nq);
  f.args.nkv = static_cast<int>(nkv);
  f.args.Tmax = static_cast<int>(kc.size(-2));
  f.args.head_dim = D;
  f.args.eps = static_cast<float>(eps);
  dec_gemm_run(x, w, f);
  return q;
}

std::tuple<at::Tensor, at::Tensor> dec_gemm_residual_norm(at::Tensor x, at::Tensor w, at::Tensor residual, at::Tensor nw,
                                                          double eps) {
  const int64_t H = w.size(0);
  TORCH_CHECK(residual.is_contiguous() && residual.size(0) == x.size(0) && residual.size(1) == H,
              "dec_gemm_residual_norm: residual shape");
  TORCH_CHECK(H % 8 == 0 && H <= 8 * 192 * 4, "dec_gemm_residual_norm: width");
  const c10::cuda::CUDAGuard g(x.device());
  at::Tensor h = at::empty_like(residual), hn = at::empty_like(residual);
  DecFuse f{};
  f.consumer = DEC_RESNORM;
  f.args.res = reinterpret_cast<const bf16_t*>(residual.data_ptr());
  f.args.nw = reinterpret_cast<const bf16_t*>(nw.data_ptr());
  f.args.h_out = reinterpret_cast<bf16_t*>(h.data_ptr());
  f.args.hn_out = reinterpret_cast<bf16_t*>(hn.data_ptr());
  f.args.eps = static_cast<float>(eps);
  dec_gemm_run(x, w, f);
  return {h, hn};
}

at::Tensor dec_gemm_swiglu(at::Tensor x, at::Tensor w) {
  TORCH_CHECK(w.size(0) % 16 == 0, "dec_gemm_swiglu: width must be a multiple of 16");
  const c10::cuda::CUDAGuard g(x.device());
  at::Tensor act = at::empty({x.size(0), w.size(0) / 2}, x.options());
  DecFuse f{};
  f.consumer = DEC_SWIGLU;
  f.args.act = reinterpret_cast<bf16_t*>(act.data_ptr());
  dec_gemm_run(x, w, f);
  return act;
}

// Stream-K partials with per-CTA phase timestamps written to ``trace`` (int64 [>= grid * 8]): a measurement
// aid for the decode GEMM's fixed latency.
static std::tuple<at::Tensor, std::vector<int64_t>> tcgen05_partials(const at::Tensor& A, const at::Tensor& B);

std::tuple<at::Tensor, std::vector<int64_t>> gemm_partials_traced(at::Tensor A, at::Tensor B, at::Tensor trace) {
  TORCH_CHECK(trace.scalar_type() == at::kLong && trace.is_cuda() && trace.numel() >= 148 * 8, "trace: int64 [grid*8]");
  g_trace = reinterpret_cast<unsigned long long*>(trace.data_ptr());
  auto out = tcgen05_partials(A, B);
  g_trace = nullptr;
  return out;
}

// Decode-shaped partial sums: the skinny mma.sync kernel (decode_gemm.cu) for M <= 64 when
// VLMRL_SKINNY_GEMM=1, else the stream-K tcgen05 kernel; both write the same [slots, M, N] layout.
std::tuple<at::Tensor, std::vector<int64_t>> gemm_partials(at::Tensor A, at::Tensor B) {
  if (skinny_enabled() && A.size(0) <= 64 && A.size(1) % 8 == 0 && B.size(0) % 8 == 0)
    return skinny_partials(A, B, g_static_weights);
  return tcgen05_partials(A, B);
}

static std::tuple<at::Tensor, std::vector<int64_t>> tcgen05_partials(const at::Tensor& A, const at::Tensor& B) {
  at::Tensor ws;
  SkMeta m{};
  gemm_ex(A, B, at::Tensor(), at::Tensor(), at::Tensor(), at::Tensor(), true, true, 1.0, EPI_STORE, false, nullptr, 0,
          &ws, &m);
  return {ws, {m.M, m.N, m.tiles_m, m.tiles_n, m.kb_count, m.grid, m.bm, m.bn}};
}

}  // namespace vlm

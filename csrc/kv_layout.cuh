// Where a token's key / value row lives in one layer's KV cache.
//
// Contiguous cache: [B, Hkv, Tmax, D], row (b, h, t) at ((b * Hkv + h) * Tmax + t).
// Paged cache: a pool of kKvBlock-token blocks [NB, Hkv, kKvBlock, D] and a block table [B, mb] of pool
// block ids; token t of sequence b is in block table[b][t / kKvBlock] at offset t % kKvBlock.  Sequences
// may share blocks (a GRPO group's members point at their leader's full prompt blocks), so a block's
// contents are read through any table row that names it.  A 64-key attention chunk that starts on a
// multiple of kKvBlock lies inside one block, so a tiled TMA box still covers it.
#pragma once

#include <ATen/ATen.h>
#include <c10/util/Optional.h>

#include "common.cuh"

namespace vlm {

constexpr int kKvBlock = 64;

struct KvLayout {
  const int* table;  // nullptr: contiguous
  int mb;            // block-table row stride (blocks per sequence)
  int T;             // rows per (sequence or block, head): Tmax (contiguous) or kKvBlock (paged)
  int Hkv;
  int cap;           // token capacity per sequence: Tmax or mb * kKvBlock
};

__host__ __device__ inline int64_t kv_row(const KvLayout& a, int b, int h, int t) {
  if (a.table == nullptr) return (static_cast<int64_t>(b) * a.Hkv + h) * a.T + t;
  const int blk = a.table[static_cast<int64_t>(b) * a.mb + t / kKvBlock];
  return (static_cast<int64_t>(blk) * a.Hkv + h) * kKvBlock + (t % kKvBlock);
}

// Host: the layout of cache layer `kc` ([B, Hkv, Tmax, D], or the pool [NB, Hkv, kKvBlock, D] with `table`
// int32 [B, mb]).
inline KvLayout kv_layout_of(const at::Tensor& kc, const c10::optional<at::Tensor>& table) {
  TORCH_CHECK(kc.dim() == 4 && kc.is_contiguous(), "KV cache layer: contiguous [rows, Hkv, T, D]");
  KvLayout a{};
  a.Hkv = static_cast<int>(kc.size(1));
  if (table.has_value() && table->defined()) {
    const at::Tensor& t = *table;
    TORCH_CHECK(t.scalar_type() == at::kInt && t.dim() == 2 && t.is_contiguous() && t.device() == kc.device(),
                "block table: contiguous int32 [B, blocks] on the cache's device");
    TORCH_CHECK(kc.size(2) == kKvBlock, "paged KV pool: blocks of ", kKvBlock, " tokens");
    a.table = t.data_ptr<int>();
    a.mb = static_cast<int>(t.size(1));
    a.T = kKvBlock;
    a.cap = a.mb * kKvBlock;
  } else {
    a.table = nullptr;
    a.mb = 0;
    a.T = static_cast<int>(kc.size(2));
    a.cap = a.T;
  }
  return a;
}

}  // namespace vlm

// Python bindings of the vlmrl sm_100a kernels (module vlmrl._C).
#include <torch/extension.h>

#include "host_utils.h"
#include "vlm_ops.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "vlmrl hand-written sm_100a kernels";
  m.def("gemm", &vlm::gemm, "tcgen05 GEMM with fused epilogues");
  m.def("gemm_gather", &vlm::gemm_gather, "tcgen05 GEMM whose weight operand is all-gathered from peer shards in-kernel");
  m.def("unit_gather", &vlm::unit_gather, "copy byte ranges of a sharded unit from the peers' shards");
  m.def("dec_gemm_qkv", &vlm::dec_gemm_qkv, "decode qkv GEMM with the q/k norm + RoPE + KV append consumer fused");
  m.def("dec_gemm_residual_norm", &vlm::dec_gemm_residual_norm, "decode GEMM with residual + RMSNorm fused");
  m.def("dec_gemm_swiglu", &vlm::dec_gemm_swiglu, "decode gate/up GEMM with SwiGLU fused");
  m.def("gemm_partials", &vlm::gemm_partials, "stream-K partial sums for the fused decode consumers");
  m.def("gemm_partials_traced", &vlm::gemm_partials_traced, "gemm_partials with per-CTA phase timestamps");
  m.def("set_static_weights", &vlm::set_static_weights);
  m.def("dec_qkv", &vlm::dec_qkv, py::arg("ws"), py::arg("meta"), py::arg("bias"), py::arg("qw"), py::arg("kw"),
        py::arg("lengths"), py::arg("delta"), py::arg("inv_freq"), py::arg("kc"), py::arg("vc"), py::arg("nq"),
        py::arg("nkv"), py::arg("eps"), py::arg("prefetch") = py::none(), py::arg("block_table") = py::none());
  m.def("dec_residual_norm", &vlm::dec_residual_norm, py::arg("ws"), py::arg("meta"), py::arg("residual"), py::arg("w"),
        py::arg("eps"), py::arg("prefetch") = py::none());
  m.def("dec_swiglu", &vlm::dec_swiglu, py::arg("ws"), py::arg("meta"), py::arg("prefetch") = py::none());
  m.def("tp_step_begin", &vlm::tp_step_begin, "advance the tensor-parallel decode epoch (device counter)");
  m.def("dec_residual_norm_tp", &vlm::dec_residual_norm_tp,
        "residual + RMSNorm consumer that all-reduces row-parallel partials over NVLink (tagged 8-byte words "
        "stored into every rank's slot, no fence or flag)");
  m.def("rms_norm_fwd", &vlm::rms_norm_fwd);
  m.def("rms_norm_bwd", &vlm::rms_norm_bwd);
  m.def("layer_norm_fwd", &vlm::layer_norm_fwd);
  m.def("qk_norm_rope_fwd", &vlm::qk_norm_rope_fwd);
  m.def("qk_norm_rope_bwd", &vlm::qk_norm_rope_bwd);
  m.def("vision_rope", &vlm::vision_rope, py::arg("qkv"), py::arg("rc"), py::arg("q"), py::arg("k"), py::arg("v"),
        py::arg("n_heads"), py::arg("style") = 0);
  m.def("swiglu_bwd", &vlm::swiglu_bwd);
  m.def("embed", &vlm::embed);
  m.def("scatter_rows", &vlm::scatter_rows);
  m.def("embed_bwd", &vlm::embed_bwd);
  m.def("kv_write", &vlm::kv_write, py::arg("k"), py::arg("v"), py::arg("kc"), py::arg("vc"), py::arg("seq"),
        py::arg("pos"), py::arg("block_table") = py::none());
  m.def("adamw", &vlm::adamw);
  m.def("sq_norm_acc", &vlm::sq_norm_acc);
  m.def("patchify", &vlm::patchify);
  m.def("flash_attn_fwd", &vlm::flash_attn_fwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("cu"), py::arg("o"),
        py::arg("lse"), py::arg("max_seqlen"), py::arg("causal"), py::arg("scale"), py::arg("pre") = py::none());
  m.def("flash_attn_bwd", &vlm::flash_attn_bwd, py::arg("dout"), py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"),
        py::arg("lse"), py::arg("cu"), py::arg("dq"), py::arg("dk"), py::arg("dv"), py::arg("max_seqlen"),
        py::arg("causal"), py::arg("scale"), py::arg("pre") = py::none(), py::arg("xq") = py::none());
  m.def("decode_attn", &vlm::decode_attn, py::arg("q"), py::arg("kc"), py::arg("vc"), py::arg("lens"), py::arg("o"),
        py::arg("scale"), py::arg("prefetch") = py::none(), py::arg("lead") = py::none(),
        py::arg("share_len") = py::none(), py::arg("block_table") = py::none());
  m.def("sample", &vlm::sample);
  m.def("lm_head_sample", &vlm::lm_head_sample, "lm_head GEMM with a top-k epilogue + merge / top-p / Philox draw");
  m.def("lm_head_sample_tp", &vlm::lm_head_sample_tp,
        "vocab-parallel lm_head_sample: shard top-k survivors exchanged over NVLink as tagged words");
  m.def("vocab_logprob_fwd", &vlm::vocab_logprob_fwd);
  m.def("vocab_logprob_bwd", &vlm::vocab_logprob_bwd);
  m.def("symm_alloc", &vlm::symm_alloc, "cudaMalloc an IPC-exportable buffer");
  m.def("symm_free", &vlm::symm_free);
  m.def("symm_ipc_handle", &vlm::symm_ipc_handle);
  m.def("symm_open", &vlm::symm_open, "map a peer's buffer from its IPC handle");
  m.def("symm_close", &vlm::symm_close);
  m.def("symm_view", &vlm::symm_view);
  m.def("rs_pull", &vlm::rs_pull, "reduce-scatter by pulling shards from peer memory");
  m.def("adamw_push", &vlm::adamw_push, "sharded AdamW storing bf16 params into every rank's gathered buffer");
  m.def("peer_wait", &vlm::peer_wait, py::arg("local_sig"), py::arg("slot"), py::arg("target"), py::arg("rank"),
        py::arg("world"), py::arg("device"), py::arg("budget_cycles") = 0);
  m.def("peer_barrier", &vlm::peer_barrier);
  m.def("decode_step_maps", &vlm::decode_step_maps, "tensor maps (CPU bytes) of the persistent decode step");
  m.def("decode_step_sync_words", &vlm::decode_step_sync_words);
  m.def("decode_step_ws_floats", &vlm::decode_step_ws_floats);
  m.def("decode_step", &vlm::decode_step, "all decoder layers of one decode step in one persistent launch",
        py::arg("wmaps"), py::arg("amaps"), py::arg("layers"), py::arg("x"), py::arg("h1"), py::arg("xn"), py::arg("o"),
        py::arg("hn"), py::arg("act"), py::arg("ws"), py::arg("ssq"), py::arg("sync"), py::arg("lens"), py::arg("delta"),
        py::arg("inv_freq"), py::arg("lead") = py::none(), py::arg("share_len") = py::none(), py::arg("dims"),
        py::arg("eps"), py::arg("scale"), py::arg("trace") = py::none());
  m.def("read_and_clear_error", &vlm::read_and_clear_error);
  m.def("read_error_words", &vlm::read_error_words, "error code and detail words of a device, then cleared");
  m.def("launch_count", &vlm::launch_count, "kernel launches issued by this library so far");
}

// Rust binding of include/inferox.h (libinferox_b200.so) for the reference
// crate: copy to src/cuda/ffi.rs. Every header entry point has a
// declaration here; the types mirror the header's structs field by field.

use std::ffi::{c_char, c_int, c_void};

#[repr(C)] pub struct IfxModel { _p: [u8; 0] }
#[repr(C)] pub struct IfxKv { _p: [u8; 0] }
#[repr(C)] pub struct IfxKvBatch { _p: [u8; 0] }
#[repr(C)] pub struct IfxTokenizer { _p: [u8; 0] }
#[repr(C)] pub struct IfxQMatrix { _p: [u8; 0] }

#[repr(C)]
#[derive(Clone, Copy)]
pub struct IfxLoadOpts {
    pub device: c_int, pub tp_size: c_int, pub tp_rank: c_int,
    pub nccl_comm: *mut c_void, pub rope_compat: c_int,
    pub use_graphs: c_int, pub persistent_decode: c_int,
    pub kquant_layout: c_int,  // 0: the reference's byte semantics; 1: a llama.cpp file
    pub tp_timeout_ms: c_int,  // longest wait for a call's collectives (0: 300000)
}

#[repr(C)]
pub struct IfxConfig {
    pub vocab_size: u32,
    pub hidden_size: u64, pub n_layers: u64, pub n_heads: u64,
    pub n_kv_heads: u64, pub head_dim: u64, pub intermediate_size: u64,
    pub norm_eps: f32, pub rope_base: f32,
    pub rope_dim: u64, pub context_length: u64,
    pub architecture: [c_char; 64],
}

#[repr(C)]
pub struct IfxSampler { pub temperature: f32, pub top_k: u64, pub top_p: f32 }

#[repr(C)]
pub struct IfxSynthSpec {
    pub vocab: u32, pub dim: u32, pub n_layers: u32, pub n_heads: u32, pub n_kv_heads: u32,
    pub ffn: u32, pub context: u32,
    pub rope_base: f32, pub norm_eps: f32, pub sigma: f32,
    pub mix: c_int, pub tied: c_int, pub seed: u64, pub threads: c_int,
}

extern "C" {
    pub fn ifx_last_error() -> *const c_char;
    pub fn ifx_status_name(s: c_int) -> *const c_char;
    pub fn ifx_version() -> c_int;
    pub fn ifx_load_opts_default(o: *mut IfxLoadOpts);
    pub fn ifx_model_load(path: *const c_char, o: *const IfxLoadOpts, out: *mut *mut IfxModel) -> c_int;
    pub fn ifx_model_load_mem(bytes: *const c_void, len: usize, o: *const IfxLoadOpts,
                              out: *mut *mut IfxModel) -> c_int;
    pub fn ifx_model_decode_weight_bytes(m: *const IfxModel) -> u64;
    pub fn ifx_model_free(m: *mut IfxModel);
    pub fn ifx_model_config(m: *const IfxModel, out: *mut IfxConfig) -> c_int;
    pub fn ifx_kv_create(m: *mut IfxModel, max_seq: usize, out: *mut *mut IfxKv) -> c_int;
    pub fn ifx_kv_free(kv: *mut IfxKv);
    pub fn ifx_kv_clear(kv: *mut IfxKv) -> c_int;
    pub fn ifx_kv_len(kv: *const IfxKv) -> usize;
    pub fn ifx_kv_read(kv: *const IfxKv, layer: usize, which_v: c_int, out: *mut f32) -> c_int;
    pub fn ifx_kv_decode_kernels(kv: *const IfxKv) -> c_int;
    pub fn ifx_prefill(m: *mut IfxModel, kv: *mut IfxKv, ids: *const u32, n: usize,
                       logits: *mut f32, last_row_only: c_int) -> c_int;
    pub fn ifx_decode_step(m: *mut IfxModel, kv: *mut IfxKv, token: u32, logits: *mut f32) -> c_int;
    pub fn ifx_forward(m: *mut IfxModel, ids: *const u32, n: usize, logits: *mut f32,
                       last_row_only: c_int) -> c_int;
    pub fn ifx_generate(m: *mut IfxModel, kv: *mut IfxKv, prompt: *const u32, n_prompt: usize,
                        max_tokens: usize, out: *mut u32) -> c_int;
    pub fn ifx_sample(m: *mut IfxModel, s: *const IfxSampler, seed: u64, offset: u64,
                      out: *mut u32) -> c_int;
    pub fn ifx_decode_greedy(m: *mut IfxModel, kv: *mut IfxKv, token: u32, n_steps: usize,
                             out: *mut u32, device_ms: *mut f32) -> c_int;
    pub fn ifx_bench_matmul_t_q(a_dev: *const f32, w: *const IfxQMatrix, c_dev: *mut f32, m: usize,
                                reps: c_int, ms_per_call: *mut f32) -> c_int;
    pub fn ifx_bench_kernel(m: *mut IfxModel, kv: *mut IfxKv, which: *const c_char, reps: c_int,
                            ms_per_launch: *mut f32, bytes_per_launch: *mut u64) -> c_int;
    // batched decode: `batch` independent caches, prefilled one by one, stepped together
    pub fn ifx_kv_batch_create(m: *mut IfxModel, max_seq: usize, batch: c_int,
                               out: *mut *mut IfxKvBatch) -> c_int;
    pub fn ifx_kv_batch_create_paged(m: *mut IfxModel, max_seq: usize, batch: c_int,
                                     n_pages: usize, out: *mut *mut IfxKvBatch) -> c_int;
    pub fn ifx_kv_batch_pages(kb: *const IfxKvBatch, free_pages: *mut usize,
                              total_pages: *mut usize) -> c_int;
    pub fn ifx_kv_batch_free(kb: *mut IfxKvBatch);
    pub fn ifx_kv_batch_len(kb: *const IfxKvBatch, seq: c_int, len: *mut usize) -> c_int;
    pub fn ifx_prefill_seq(m: *mut IfxModel, kb: *mut IfxKvBatch, seq: c_int, ids: *const u32,
                           n: usize, logits: *mut f32, last_row_only: c_int) -> c_int;
    pub fn ifx_decode_step_batch(m: *mut IfxModel, kb: *mut IfxKvBatch, tokens: *const u32,
                                 logits: *mut f32, argmax: *mut u32) -> c_int;
    pub fn ifx_decode_greedy_batch(m: *mut IfxModel, kb: *mut IfxKvBatch, tokens: *const u32,
                                   n_steps: usize, out: *mut u32, device_ms: *mut f32) -> c_int;
    // op level: device pointers + a cudaStream_t (null = default stream)
    pub fn ifx_op_dequantize(ty: c_int, bytes: *const c_void, nbytes: usize, out: *mut f32,
                             n_out: usize, stream: *mut c_void) -> c_int;
    pub fn ifx_op_matmul_t(a: *const f32, b: *const f32, c: *mut f32, m: usize, n: usize,
                           k: usize, stream: *mut c_void) -> c_int;
    pub fn ifx_op_matmul(a: *const f32, b: *const f32, c: *mut f32, m: usize, n: usize,
                         k: usize, stream: *mut c_void) -> c_int;
    pub fn ifx_qmatrix_create(ty: c_int, gguf_bytes: *const c_void, nbytes: usize, rows: usize,
                              cols: usize, device: c_int, out: *mut *mut IfxQMatrix) -> c_int;
    pub fn ifx_qmatrix_free(w: *mut IfxQMatrix);
    pub fn ifx_op_matmul_t_q(a: *const f32, w: *const IfxQMatrix, c: *mut f32, m: usize,
                             stream: *mut c_void) -> c_int;
    pub fn ifx_op_silu(x: *mut f32, n: usize, stream: *mut c_void) -> c_int;
    pub fn ifx_op_embedding_lookup(emb: *const f32, emb_len: usize, ids: *const u32, n_ids: usize,
                                   hidden: usize, out: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ifx_op_rms_norm_rows(x: *mut f32, w: *const f32, eps: f32, rows: usize, hidden: usize,
                                stream: *mut c_void) -> c_int;
    pub fn ifx_op_rope(x: *mut f32, seq: usize, heads: usize, d: usize, rope_dim: usize,
                       base: f32, pos0: usize, stream: *mut c_void) -> c_int;
    pub fn ifx_op_softmax_rows(x: *mut f32, rows: usize, cols: usize, stream: *mut c_void) -> c_int;
    pub fn ifx_op_swiglu(g: *const f32, u: *const f32, out: *mut f32, n: usize,
                         stream: *mut c_void) -> c_int;
    pub fn ifx_op_add_in_place(out: *mut f32, b: *const f32, n: usize, stream: *mut c_void) -> c_int;
    pub fn ifx_op_argmax(x: *const f32, n: usize, out: *mut u32, stream: *mut c_void) -> c_int;
    pub fn ifx_op_sample_u(logits: *const f32, n: usize, s: *const IfxSampler, u: f32,
                           token_host: *mut u32, stream: *mut c_void) -> c_int;
    pub fn ifx_op_sample_u_static(logits: *const f32, n: usize, s: *const IfxSampler, u: f32,
                                  token_dev: *mut u32, stream: *mut c_void) -> c_int;
    // tensor parallelism: a communicator made by the library's own NCCL instance
    pub fn ifx_tp_unique_id(id_out: *mut u8) -> c_int;  // 128 bytes, on rank 0
    pub fn ifx_tp_comm_create(id: *const u8, nranks: c_int, rank: c_int, device: c_int,
                              comm_out: *mut *mut c_void) -> c_int;
    pub fn ifx_tp_comm_destroy(comm: *mut c_void);
    pub fn ifx_tp_shard(ty: c_int, gguf_bytes: *const c_void, nbytes: usize, rows: usize,
                        cols: usize, split_k: c_int, tp: c_int, rank: c_int, out: *mut c_void,
                        out_bytes: *mut usize) -> c_int;
    pub fn ifx_decode_step_batch_seqs(m: *mut IfxModel, kb: *mut IfxKvBatch, seqs: *const c_int,
                                      n: c_int, tokens: *const u32, logits: *mut f32,
                                      argmax: *mut u32) -> c_int;
    pub fn ifx_kv_batch_reset(m: *mut IfxModel, kb: *mut IfxKvBatch, seq: c_int) -> c_int;
    pub fn ifx_kquant_from_ggml(ggml_type: u32, src: *const c_void, nbytes: usize, dst: *mut c_void,
                                type_out: *mut c_int, signed_scales_out: *mut c_int) -> c_int;
    // tokenizer (src/tokenizer/mod.rs): host code, no GPU needed
    pub fn ifx_tokenizer_load(path: *const c_char, out: *mut *mut IfxTokenizer) -> c_int;
    pub fn ifx_tokenizer_load_json(json: *const c_char, len: usize,
                                   out: *mut *mut IfxTokenizer) -> c_int;
    pub fn ifx_tokenizer_free(t: *mut IfxTokenizer);
    pub fn ifx_tokenizer_encode(t: *const IfxTokenizer, text: *const c_char, len: usize,
                                ids: *mut u32, cap: usize, n_ids: *mut usize) -> c_int;
    pub fn ifx_tokenizer_decode(t: *const IfxTokenizer, ids: *const u32, n: usize,
                                text: *mut c_char, cap: usize, len: *mut usize) -> c_int;
    pub fn ifx_tokenizer_vocab_size(t: *const IfxTokenizer, n: *mut usize) -> c_int;
    // synthetic workloads (the benchmark models and test fixtures)
    pub fn ifx_synth_gguf(spec: *const IfxSynthSpec, bytes_out: *mut *mut c_void,
                          len_out: *mut usize) -> c_int;
    pub fn ifx_synth_free(bytes: *mut c_void);
    pub fn ifx_quantize(ty: c_int, x: *const f32, n: usize, out: *mut c_void) -> c_int;
    pub fn ifx_synth_normal(seed: u64, stream: u64, sigma: f32, out: *mut f32, n: usize) -> c_int;
}

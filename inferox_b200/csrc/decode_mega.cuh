// Persistent batch-1 decode step: the whole token (embedding, every layer,
// logits, argmax) in one cooperative launch of one CTA per SM.
#pragma once
#include "gemv.cuh"

namespace ifx {

enum MegaKind { PH_EMBED = 0, PH_GEMV = 1, PH_ATTN = 2, PH_ARGMAX = 4, PH_ALLREDUCE = 5 };

constexpr int kMaxRanks = 8;

struct MegaAttn {
  __half *kc, *vc;  // this layer's caches [G][max_seq][hd]
  int layer;
};

// 16-byte aligned (and so a multiple of 16 in size): the kernel moves
// records into shared memory with bulk async copies.
struct __align__(16) MegaPhase {
  int kind;
  GemvArgs g;   // PH_GEMV (sched has one entry per CTA)
  MegaAttn at;  // PH_ATTN
  float *zero_ptr;  // buffer this phase zeroes (a later phase accumulates into it)
  int zero_n;
  int attn_prefetch;  // layer + 1 on the QKV GEMV: during it, fetch this CTA's first
                      // attention item's cached K/V rows of that layer (0: none)
  // PH_ALLREDUCE (tensor parallelism): ar_dst[i] += sum over ranks of their
  // ar_src[i] (i < ar_n); ar_src is left zeroed. ar_index counts the
  // all-reduces of the step from 1.
  float *ar_src, *ar_dst;
  int ar_n, ar_index;
};

// Tensor parallelism inside the persistent kernel: every rank owns one
// buffer that all ranks map (CUDA IPC), laid out as
//   recv  [2][kMaxRanks][row_floats] u64  elements pushed by each rank, two
//                                        parities: epoch << 32 | f32 bits
//   (off_flags) [grid][kMaxRanks] u32    reserved
//   keys  [2][kMaxRanks] u64            each rank's argmax key, two parities
//   kflags [kMaxRanks] u32               epoch of rank r's last key
// Epochs only grow (counters in `epoch`, advanced by the kernel itself), so
// nothing is ever reset between steps.
struct MegaPeers {
  char *buf[kMaxRanks];  // rank r's buffer as mapped in this process (buf[rank]: own)
  size_t off_flags, off_keys, off_kflags;
  int row_floats;
  unsigned *epoch;  // [0] all-reduces so far, [1] steps so far (this rank's device memory)
  uint64_t wait_ns;  // a wait for another rank gives up (error flag) after this long
};

struct MegaArgs {
  const MegaPhase *ph;
  int nph;
  const int2 *rg;  // [grid][nph_pad]: each CTA's unit range per phase
  int nph_pad;     // nph rounded up to even (rows are 16-byte multiples)
  // dynamic shared memory carve-up (byte offsets)
  int off_ph, off_rg, off_tab, off_ring, off_scr, off_stage;  // off_scr: attention buffer
  int ring_bytes, slot_bytes, scratch_bytes;
  unsigned *bar;  // [0] grid barrier counter, [1 + h] finished splits of kv head h;
                  // all zeroed at every launch
  int *err;
  // token loop state
  const uint8_t *emb;
  int emb_type, D, V;
  uint32_t *next_token;
  float *x, *attn, *logits;
  float *part_o;
  float2 *part_ml;
  int H, G, hd, max_seq, rope_compat, rope_dim;
  // attention splits per kv head: nsa for a full cache (it sizes the item
  // buffer and the partials), at least nsa_base in any step
  int nsa, nsa_base;
  int attn_tc;  // 4 / 8: attention items on tensor cores with that many head slots (head size a multiple of 64); 0: FMA loops
  float rope_base;
  const float *qkv;
  const __half *kc0, *vc0;  // layer 0 of the K and V caches
  size_t kv_layer_elems;    // elements per layer of one cache
  int *pos;
  unsigned long long *amax_key;
  int *amax_count;
  uint32_t *tokens;
  int *n_out;
  // tensor parallelism (nranks 1: none)
  int rank, nranks, v0;  // v0: global index of this rank's first logit
  int n_ar;              // all-reduce phases per step
  MegaPeers peers;
};

struct MegaPlan {
  MegaArgs args{};
  MegaPhase *d_phases = nullptr;
  int2 *d_rg = nullptr;
  size_t smem = 0;
  int grid = 0;
};

// Attention split count for a cache of max_seq rows with G kv heads, and the
// fewest splits a step uses (the count that spreads items over the SMs).
int mega_attn_splits(int G, int max_seq, int num_sms);
int mega_attn_splits_base(int G, int num_sms);
// Shared-memory bytes the attention phase needs.
size_t mega_attn_scratch(int grp, int hd, int max_seq, int nsa);
// Bytes of one rank's peer buffer for vectors of up to n floats.
size_t mega_peer_bytes(int n, int grid, MegaPeers *layout);
ifx_status mega_finalize(MegaPlan *plan, const std::vector<MegaPhase> &phases, int num_sms);
ifx_status mega_launch(const MegaPlan &plan, cudaStream_t st);
void mega_free(MegaPlan *plan);

}  // namespace ifx

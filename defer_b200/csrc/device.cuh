// Device-side model/batch views of the token step.
//
// Every phase is written against a work partition (cta, ncta) so the same
// code runs either as one launch per phase or inside the persistent
// token-loop kernel with grid barriers between phases. The arithmetic of
// every output element is fixed by the data alone (never by the launch
// geometry, the batch size or the number of sessions in flight), so the
// single-session, batched and persistent paths are bit-identical.
//
// Canonical arithmetic (all fp32, round-to-nearest):
//  * dot(w_row, x): the row is cut into 16-byte chunks (4 fp32 or 8 bf16
//    weights); chunk j belongs to lane j % 32; each lane accumulates its
//    chunks in increasing j with fmaf in element order; the 32 lane partials
//    are combined by an xor butterfly (offsets 16, 8, 4, 2, 1).
//  * rmsnorm: ss = dot(x, x) with the fp32 rule; inv = 1 / sqrt(ss/n + eps);
//    out = (x * inv) * w (ops.rs:84-95 order).
//  * RoPE: host-built cos/sin tables (model.rs:438-445 bit-exact), rotation
//    without contraction (model.rs:446-456).
//  * attention: keys in fixed chunks of kAttnChunk positions. Score =
//    ((a0 + a1) + (a2 + a3)) * scale with a_c = fmaf chain over d % 4 == c;
//    per chunk m = max, e = expf(s - m), l = butterfly tree over the 64 slots,
//    acc[d] = fmaf chain over t; chunks combined in order:
//    w_c = expf(m_c - M), L = fmaf(w_c, l_c, L), O = fmaf(w_c, acc_c, O),
//    out = O / L.
//  * SiLU/GeLU, residual add: no contraction, ops.rs:120-156 order.
//  * sampler (sampler.rs:24-109): argmax exact (NaN skipped, lowest index on
//    ties); s = l / T, M = max s, e = expf(s - M), Z = e_0 + e_1 + ... and
//    the CDF over p = e * (1/Z) as the reference's sequential fp32 sums,
//    reproduced bit for bit by integer runs inside one binade (phases.cuh,
//    exact sampler); only expf itself may differ from the reference's libm.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace defer {

constexpr int kThreads = 256;       // threads per CTA for every phase
constexpr int kWarps = kThreads / 32;
constexpr int kAttnChunk = 64;      // key positions per attention chunk
constexpr int kSBlk = 32;           // sampler block: elements per block (one per lane)
constexpr int kMaxGroup = 8;        // slots per register tile of the dataflow kernel
constexpr int kMaxGroupWide = 32;   // slots per register tile of the grid-barrier / per-phase kernels

enum StatusCode : int {
  kStOk = 0,
  kStDivergence = 1,   // recorded token differs from the re-sampled one
  kStTimeout = 2,      // a grid barrier gave up waiting
  kStBadToken = 3,     // token id out of range
  kStContext = 4,      // context length exceeded
};

struct DLayer {
  const float* attn_norm;
  const void* wqkv;   // [QD + 2 KVD, H], rows pair-interleaved
  const float* bqkv;  // [QD + 2 KVD] or null, same order
  const void* wo;     // [H, QD]
  const float* ffn_norm;
  const void* wgu;    // [2 FF, H], row 2j = gate_j, row 2j+1 = up_j
  const void* wdown;  // [H, FF]
};

struct DModel {
  int V, H, FF, L, NH, NKV, HD, HALF, QD, KVD, QKVR, max_seq;
  float eps, scale;
  int gelu, bf16, bias;
  const void* embed;     // [V, H]
  const void* head;      // [V, H] (aliases embed when tied)
  const float* norm;     // [H]
  const float* rope_cos;  // [max_seq, HALF]
  const float* rope_sin;
  const DLayer* layers;  // device array [L]
};

// Per-session program for a run of steps. Step s of session b:
//   s <  n_prompt           : feed tokens[s]
//   n_prompt <= s < n_total : sample (T > 0 draws words[s - n_prompt]);
//                             verify mode compares with tokens[s] and feeds
//                             tokens[s]; generate mode feeds the sample and
//                             stores it in tokens[s]
struct DSession {
  float* kc;              // [L][NKV][cap][HD]
  float* vc;
  const uint32_t* mask;   // [cap/32 + 1] bitmap of masked positions, or null
  uint32_t* tokens;       // [n_total]
  const uint32_t* words;  // [n_total - n_prompt] PRNG words (T > 0)
  float* margins;         // [n_total - n_prompt] sampler margins, or null
  const uint32_t* stop;   // stop tokens (generate mode)
  int n_stop;
  int cap;
  int pos;                // cache length at the start of the run
  int n_prompt, n_total;
  float temperature;
  int verify;             // 1: replay/checkout, 0: generate
  // Position-parallel replay (verify mode): `lanes` slots share one cache
  // and program; the slot whose first step index is j feeds the indices
  // j, j + lanes, j + 2 lanes, ..., and from the logits of index i it
  // verifies the token of index i + 1 in its next step. 1 otherwise.
  int lanes;
};

// Mutable per-slot state written by the kernels.
struct DSlotState {
  int pos;        // current cache length
  int step;       // next step index
  int active;     // 1 while this slot is feeding a token in the current step
  int done;       // program finished (or stopped)
  int was_active;
  uint32_t cur;   // token being fed in the current step
  int div_step;   // first diverging step (verify mode), -1 if none
  uint32_t div_token;
};

// Sampler block statistics of one slot (nblk = ceil(V / kSBlk) entries each).
struct DSampleStats {
  float* lmax;   // [B][nblk] largest raw logit of the block (NaN skipped)
  int* larg;     // [B][nblk] its index (lowest on ties), INT_MAX if none
  float* smax;   // [B][nblk] largest s = l / T of the block
  float* esum;   // [B][nblk] block sums of e
  float* psum;   // [B][nblk] block sums of p
};

struct DBatch {
  int B;
  const DSession* sess;   // [B]
  DSlotState* st;         // [B]
  float* x;               // [B, H] residual stream
  float* q;               // [B, QD]
  float* att;             // [B, QD]
  float* g;               // [B, FF]
  float* logits;          // [B, V]
  float* part;            // [B, NH, max_chunks, HD + 2] attention partials
  int* tickets;           // [B, NKV] attention chunks finished (last one combines)
  int max_chunks;
  int nblk;               // sampler blocks per slot
  DSampleStats ss;
  int* status;            // global status word
  int* any_active;        // [2] set by the select phase (indexed by step parity)
  unsigned* bar;          // grid barrier counter
  unsigned smem_bytes;    // dynamic shared memory of the launch (stages copy
                          // their weight rows into what their inputs leave free)
  int parts;              // wide projections: CTA partitions, each owning every
                          // parts-th slot group and all rows of the matrix
  // Instrumentation and fault drills; all zero in normal runs.
  unsigned long long* trace;  // [ncta][stages][kTraceSlots] globaltimer stamps of step
  int trace_step;             //   trace_step (dataflow kernel), or null
  int stall;                  // 1: CTA 0 withholds its first hand-off of step 0
  unsigned long long wait_ns; // limit of every bounded wait (0: the kernel's default)
};

// Trace record of one stage of one CTA (dataflow kernel): slot 0 = stage
// entry, 1 = inputs received (after the poll), 2 + w = warp w done; warp 0
// also marks 10 = RMS statistic ready / attention rows staged / sampler
// started, 11 = first weight piece in shared memory / attention scores
// done / token sampled, 12 = attention softmax done / sampler sum records
// published, 13 = attention weighted sum done / sum walked, 14 = attention
// units done / CDF records published, 15 = attention combines done / CDF
// walked; SELECT's owner also marks 16 / 19 = sum / CDF records polled,
// 17 / 20 = decoded and crossed rows loaded, 18 / 21 = walk done.
constexpr int kTraceSlots = 24;

}  // namespace defer

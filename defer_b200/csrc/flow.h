// Host entry points of the dataflow token-loop kernel (csrc/flow.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "device.cuh"

namespace defer {

// Tagged words: one fp32 value (low 32 bits) and the tag of the stage that
// wrote it (high 32 bits). Every buffer is [slot]-major.
struct FlowBufs {
  uint64_t* xt;    // [B][xw]: residual x (H words), step info (2), RoPE cos/sin (2 HALF), padding
  uint64_t* qt;    // [B][NKV][(NH/NKV + 2) HD]: per KV head its query heads, new k, new v
  uint64_t* at;    // [B][QD] attention output
  uint64_t* gt;    // [B][FF] act(gate) * up
  uint64_t* pt;    // [B][NH][max_chunks][HD + 2] attention chunk partials (m, l, acc)
  uint64_t* cl;    // [B][cta_cap][2] per-CTA greedy best (value, index bits)
  uint64_t* csm;   // [B][cta_cap] per-CTA max of s = l / T
  uint64_t* esum;  // [B][2][nblk] floats, not tagged: per logits row the max of s, the sum of exp(s - max)
  uint64_t* zrec;  // [B][nblk][2] exact sampler: per row its binade and increments in the sum of e
  uint64_t* crec;  // [B][nblk][2] the same in the CDF of p
  uint64_t* invw;  // [B] 1 / (sum of e) of a sampling slot
  int xw;          // words per slot of xt
  int cta_cap;     // CTA capacity of cl / csm
  uint32_t epoch;  // first tag of this run
};

// Shared-memory geometry of one launch.
struct FlowGeo {
  int grid;        // CTAs (one per SM, at most one per logits block)
  int ring_slots;  // weight ring: slots of slot_bytes each
  int slot_bytes;
  int stage_f;     // floats of the staging area
  int ol_f;        // floats of own logits per slot
  int ox_f;        // floats of own residual rows per slot
  int rope_f;      // floats of RoPE rows per slot
  int res_f;       // floats of the norm-weight row (H rounded up to 4)
  size_t smem_bytes;
};

struct FlowPlan {
  bool ok = false;
  const char* why = "";
  FlowGeo geo{};
};

// Whether (and how) the dataflow kernel runs a batch of B slots whose
// caches hold at most max_chunks attention chunks on a GPU with `sms` SMs.
FlowPlan flow_plan(const DModel& m, int B, int max_chunks, int sms);

// 64-bit words of every tagged buffer for B slots.
size_t flow_tagged_words(const DModel& m, int B, int max_chunks, int sms);

// Stages of one token step (the trace's second dimension).
int flow_stages_per_step(const DModel& m);

// Tags one run of nsteps steps consumes.
uint64_t flow_tags_per_run(const DModel& m, int nsteps);

// Lays the tagged buffers out in `words` (flow_tagged_words entries).
FlowBufs flow_bufs(const DModel& m, int B, int max_chunks, int sms, uint64_t* words);

void launch_steps_flow(const DModel& m, const DBatch& bt, const FlowBufs& fb, const FlowPlan& plan, int nsteps,
                       cudaStream_t st);

}  // namespace defer

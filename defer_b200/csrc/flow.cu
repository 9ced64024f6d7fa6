// Dataflow token loop: every phase of up to `nsteps` token steps of a small
// batch (B <= kMaxGroup slots) in one cooperative launch, with no grid
// barrier. Same phases and the same arithmetic as the phase kernels
// (csrc/phases.cuh: model.rs:394-520 forward, sampler.rs:78-109 sampling,
// engine.rs:62-137 / 241-274 token loop), so its results are bit-identical
// to theirs.
//
// Cross-CTA data. Every value another CTA needs travels as a tagged word:
// 8 bytes holding the fp32 value and the tag of the stage that wrote it,
// stored and loaded as one 64-bit access (single-copy atomic). A consumer
// polls the words it needs until every tag equals the stage's tag, so data
// and readiness arrive together: one L2 round trip per dependency instead
// of a barrier followed by a reload. Tags grow monotonically within a run
// (step s, stage k -> epoch + (s + 1) * stages_per_step + k) and across runs
// (the runner's epoch), so a stale word never looks ready.
//
// Overwrite safety. A CTA reads words other CTAs wrote in a stage only if it
// writes part of that stage's successor output, and every stage waits for
// all writers of the stage before it; so by the time any writer overwrites a
// buffer, every reader of its previous contents has finished. The residual
// rows a CTA owns (O and down projections) stay in its shared memory and
// only the owner rewrites them. Every CTA owns at least one logits block
// (grid <= blocks), so every CTA is on that chain once per step and none can
// fall a whole step behind.
//
// Weights. A ninth warp (the producer) streams this CTA's rows of every
// matrix, in the order the phases consume them, into a ring of shared-memory
// slots with cp.async.bulk, completion signalled on mbarriers. Weights do
// not depend on activations, so it runs ahead across phases and steps
// (bounded by the ring) and the phase warps find their rows in shared memory
// when their inputs arrive.
//
// The two plain (untagged) buffers read across CTAs:
//  * KV cache: after its QKV stage appended K/V rows, every thread of an
//    appending CTA executes fence.release.gpu at the start of its down stage
//    of that layer (after the stage barriers in between), so its
//    down-projection words, and every later tagged word, release the
//    appends. Every CTA owns down rows, whose words every CTA polls in its
//    next QKV stage; a fence.acquire.gpu after that poll acquires all
//    appends of earlier steps, and attention loads the cached rows before
//    (and while) the new q/k/v are polled.
//  * logits: every p-sum writer executes fence.release.gpu (after CTA
//    barriers that follow the logits stores) before storing its p-sums; the
//    select phase polls the p-sums, fences (acquire) and then reads the
//    chosen block's logits.
//
// Every wait is bounded: a poll or mbarrier wait past its limit, or one that
// sees another CTA's failure in the status word, marks the CTA failed; its
// phase threads leave at the next stage boundary, the producer stops issuing
// and waits for its copies in flight, and the kernel returns with the status
// word set.
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>

#include "common.h"
#include "flow.h"

// Warps 0..6 run the phases; warp 7 streams weights and takes no part in
// their barriers. Eight warps per CTA leave every thread up to 255
// registers (a ninth warp would cap them at 168 and force spills).
#define DEFER_PHASE_THREADS 224
#define DEFER_CTA_SYNC() asm volatile("bar.sync 1, 224;" ::: "memory")
#include "phases.cuh"

namespace defer {
namespace {

constexpr int kProducerWarp = kPW;       // the weight producer
constexpr int kFlowThreads = kPT + 32;
constexpr int kMaxRing = 8;
constexpr int kPollBatch = 5;    // words one thread has in flight per poll round (more spills registers)
constexpr int kCombineBatch = 10;  // the same for the attention combine (its poll site holds little else)
constexpr int kNormRegs = 19;    // norm weights held per thread (H <= 19 * 224 = 4256)
constexpr int kKvBatch = 5;      // float4 K (and V) loads one thread has in flight (5 * 224 >= 64 rows * 16)
constexpr int kStopCache = 8;    // stop tokens per slot kept in shared memory
constexpr int kSlotBytesMin = 32 * 1024;
constexpr size_t kStaticSmemReserve = 4096;
constexpr unsigned long long kWaitNs = 2000000000ull;           // phase-thread waits
constexpr unsigned long long kProducerWaitNs = 10000000000ull;  // producer waits (outlast any phase wait)

// Stage ids of a step.
__host__ __device__ constexpr int sid_qkv(int l) { return 1 + 5 * l; }
__host__ __device__ constexpr int sid_att(int l) { return 2 + 5 * l; }
__host__ __device__ constexpr int sid_o(int l) { return 3 + 5 * l; }
__host__ __device__ constexpr int sid_gu(int l) { return 4 + 5 * l; }
__host__ __device__ constexpr int sid_dn(int l) { return 5 + 5 * l; }
__host__ __device__ constexpr int sid_head(int L) { return 1 + 5 * L; }
__host__ __device__ constexpr int sid_s1(int L) { return 2 + 5 * L; }
__host__ __device__ constexpr int sid_s2(int L) { return 3 + 5 * L; }
__host__ __device__ constexpr int stages_per_step(int L) { return 4 + 5 * L; }

int group_of(int B) { return B <= 1 ? 1 : B <= 2 ? 2 : B <= 4 ? 4 : 8; }

// Words per slot of the step header (x, step info, RoPE rows), a multiple
// of 4 so every staged row starts on a 16-byte boundary.
int header_words(const DModel& m) { return (m.H + 2 + 2 * m.HALF + 3) & ~3; }

// ------------------------------------------------------------- PTX helpers
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_word(uint64_t* p, uint32_t bits, uint32_t tag) {
  const uint64_t w = ((uint64_t)tag << 32) | bits;
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ void st_f(uint64_t* p, float v, uint32_t tag) { st_word(p, __float_as_uint(v), tag); }

__device__ __forceinline__ uint64_t ld_word(const uint64_t* p) {
  uint64_t w;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
// Two adjacent words (16-byte aligned) in one load; each word is still a
// single-copy-atomic 8-byte access.
__device__ __forceinline__ void ld_word2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// One-directional gpu-scope fences: an acquire fence after relaxed reads
// that observed a release pattern orders this thread's later accesses after
// them (it does not wait for this thread's own earlier stores); a release
// fence before relaxed stores orders this thread's earlier writes before them.
__device__ __forceinline__ void fence_acquire_gpu() { asm volatile("fence.acquire.gpu;" ::: "memory"); }
__device__ __forceinline__ void fence_release_gpu() { asm volatile("fence.release.gpu;" ::: "memory"); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Global -> this CTA's shared memory bulk copy; 16-byte aligned, size % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// The same with an L2 eviction policy (createpolicy): the layers' weights
// pass through L2 once per token and go first; lm_head rows are kept, so
// that across tokens they are read from L2 rather than HBM.
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, unsigned bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Ampere-style asynchronous 16-byte copy global -> shared (no registers).
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ---------------------------------------------------------- CTA state
struct FlowShared {
  uint64_t full[kMaxRing];
  uint64_t empty[kMaxRing];
  int stop;   // the phase threads have left: the producer stops issuing
  int fail;   // a wait of a phase thread gave up, or another CTA failed
              // (written by phase threads only, read after a phase barrier)
  int pfail;  // the producer gave up (ends the phase threads' ring waits)
  int go, step, sampn;
  uint32_t tok;
  unsigned long long wait_ns;  // limit of the phase threads' bounded waits
  int act[kMaxGroup], pos[kMaxGroup], samp[kMaxGroup];
  float inv[kMaxGroup], M[kMaxGroup], Z[kMaxGroup];
  float wv[kPW][kMaxGroup];
  int wi[kPW][kMaxGroup];
  float ws[kPW][kMaxGroup];
  // Per-slot programs and state, copied in at launch: the hot path never
  // chases a pointer through global memory (L1 is mostly given to shared
  // memory). Each slot's owner CTA updates its state and writes it back.
  DSession sess[kMaxGroup];
  DSlotState st[kMaxGroup];
  uint32_t stops[kMaxGroup][kStopCache];
};

__device__ __forceinline__ bool failed(const FlowShared& sh) { return *(const volatile int*)&sh.fail != 0; }

__device__ __forceinline__ void flag_fail(FlowShared& sh, int* status, int code) {
  *(volatile int*)&sh.fail = 1;
  if (code != kStOk) atomicCAS(status, kStOk, code);
}

__device__ __forceinline__ int status_now(const int* status) { return *(const volatile int*)status; }

// The producer's failure: recorded in the status word and in its own flag,
// never in `fail`, which the phase threads must all read alike.
__device__ __forceinline__ void producer_fail(FlowShared& sh, int* status) {
  *(volatile int*)&sh.pfail = 1;
  atomicCAS(status, kStOk, kStTimeout);
}

// ------------------------------------------------- distributed sampler
// Out of line (one copy, its own register budget): the records of rows
// k0..k1 of one slot's logits held in shared memory (olg: logit i at
// olg[i - k0 * 32]), published with tag tg; `pre` is the approximate
// running sum before row k0. Warp 0 of a CTA.
__device__ __noinline__ void records_rows(const float* olg, int k0, int k1, int V, float T, float M, float inv,
                                          int cdf, const float* rm, const float* rz, float pre, uint64_t* rec,
                                          float* tile, uint32_t tg) {
  const int lane = threadIdx.x & 31;
  const float scale = cdf ? inv : 1.0f;
  const SharedVals v{olg, k0 * kSBlk, T, M, inv, cdf != 0};
  const int n = min(V, k1 * kSBlk);
  for (int row0 = k0; row0 < k1; row0 += 32) {
    const int row = row0 + lane;
    const bool has = row < k1;
    float rs = 0.0f;
    if (has) {
      const float z = ld_f(rz + row);
      rs = z > 0.0f ? z * expf(ld_f(rm + row) - M) * scale : 0.0f;
    }
    float inc = rs;
    for (int off = 1; off < 32; off <<= 1) {
      const float o = __shfl_up_sync(0xffffffffu, inc, off);
      if (lane >= off) inc += o;
    }
    int e = has ? predict_binade(pre + (inc - rs), rs) : kNoBinade;
    pre += __shfl_sync(0xffffffffu, inc, 31);
    int d0, d1;
    rows_incr(v, n, row0, k1, e, tile, nullptr, &e, &d0, &d1);
    if (has) {
      if (d0 >= (1 << 25) || d1 >= (1 << 25)) d0 = d1 = 1 << 26;
      const uint32_t code = e == kNoBinade ? 255u : e == kAnyBinade ? 254u : (uint32_t)(e + 128);
      st_word(rec + (size_t)row * 2, (uint32_t)d0, tg);
      st_word(rec + (size_t)row * 2 + 1, code | ((uint32_t)(d1 - d0 + 32768) << 8), tg);
    }
  }
}

// Rows the owner's walk loads up front, and the staging floats the walk
// needs: record words, decoded rows and blocks, the stash.
constexpr int kWalkStash = 32;
__host__ __device__ constexpr size_t walk_records_floats(int V) {
  return 5 * (size_t)((V + 31) / 32) + 3 * (size_t)(((V + 31) / 32 + 31) / 32) + 32 * (size_t)kWalkStash;
}

// Out of line: the walk over every row's record (record words in smem at
// `words`, decoded into the arrays after them) for the sum of e (cdf 0) or
// the CDF search for r over slot logits lg; the values of the rows without
// a prediction (those the walk will likely cross) are loaded up front into
// a stash. Whole CTA.
__device__ __noinline__ float walk_records(float* words, int V, const float* lg, float T, float M, float inv, int cdf,
                                           float r, int* hit, float* prev, float* at, unsigned long long* marks) {
  const int R = (V + kSBlk - 1) / kSBlk, NB = (R + 31) / 32;
  int* re = reinterpret_cast<int*>(words + 2 * R);  // [R]
  int* rd0 = re + R;                                // [R]
  int* rd1 = rd0 + R;                               // [R]
  int* be = rd1 + R;                                // [NB]
  int* bd0 = be + NB;                               // [NB]
  int* bd1 = bd0 + NB;                              // [NB]
  float* stash = reinterpret_cast<float*>(bd1 + NB);  // [kWalkStash][32]
  __shared__ int s_nstash;
  if (threadIdx.x == 0) s_nstash = 0;
  DEFER_CTA_SYNC();
  for (int row = threadIdx.x; row < R; row += kPT) {
    const uint32_t w0 = __float_as_uint(words[2 * row]), w1 = __float_as_uint(words[2 * row + 1]);
    const uint32_t code = w1 & 0xFFu;
    re[row] = code == 255u ? kNoBinade : code == 254u ? kAnyBinade : (int)code - 128;
    int slot = -1;  // a row the walk will likely cross: its values into the stash
    if (code == 255u) {
      slot = atomicAdd(&s_nstash, 1);
      if (slot >= kWalkStash) slot = -1;
    }
    rd0[row] = code == 255u ? slot : (int)w0;
    rd1[row] = (int)w0 + (int)(w1 >> 8) - 32768;
    if (slot >= 0) stash[slot * 32] = __int_as_float(row);  // the row, replaced by its values below
  }
  DEFER_CTA_SYNC();
  const SampleVals v{lg, T, M, inv, cdf != 0};
  {
    // every stashed row's 32 values in one round of loads
    const int ns = min(s_nstash, kWalkStash);
    float vals[(kWalkStash * 32 + kPT - 1) / kPT];
    int rows[(kWalkStash * 32 + kPT - 1) / kPT];
#pragma unroll
    for (int k = 0; k < (kWalkStash * 32 + kPT - 1) / kPT; k++) {
      const int f = threadIdx.x + k * kPT, sl = f >> 5;
      rows[k] = sl < ns ? __float_as_int(stash[sl * 32]) : -1;
    }
    DEFER_CTA_SYNC();
#pragma unroll
    for (int k = 0; k < (kWalkStash * 32 + kPT - 1) / kPT; k++) {
      const int f = threadIdx.x + k * kPT;
      const int i = rows[k] * 32 + (f & 31);
      vals[k] = (rows[k] >= 0 && i < V) ? v.raw(i) : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < (kWalkStash * 32 + kPT - 1) / kPT; k++) {
      const int f = threadIdx.x + k * kPT;
      if (rows[k] >= 0) stash[f] = (rows[k] * 32 + (f & 31) < V) ? v.of(vals[k]) : 0.0f;
    }
  }
  DEFER_CTA_SYNC();
  if (marks && threadIdx.x == 0) marks[0] = now_ns();
  return exact_walk(v, V, cdf != 0, r, hit, prev, at, re, rd0, rd1, be, bd0, bd1, stash, marks ? marks + 1 : nullptr,
                    reinterpret_cast<int*>(words));  // the record words are decoded: [2R] segments
}

// ------------------------------------------------------------------ polls
// A wait longer than a hand-off (the token choice of SELECT, attention on a
// few CTAs) would otherwise keep every thread of every waiting CTA
// re-reading the same few L2 lines, which slows the CTAs doing the work.
// Past kPollSpinNs of waiting a thread sleeps a quarter of the time it has
// waited beyond that between rounds (at most kPollSleepMaxNs), so a long
// wait is noticed at most ~25 % late and a short one not at all.
constexpr unsigned long long kPollSpinNs = 1500;
constexpr unsigned long long kPollSleepMaxNs = 1000;
__device__ __forceinline__ void poll_backoff(unsigned long long waited) {
  if (waited > kPollSpinNs) {
    const unsigned long long t = (waited - kPollSpinNs) >> 2;
    __nanosleep((unsigned)(t < kPollSleepMaxNs ? t : kPollSleepMaxNs));
  }
}

// One polled region: `rows` rows (only those with (mask >> r) & 1) of n
// words each, row r at src + r * sstride, its values to dst + r * dstride.
struct Seg {
  const uint64_t* src;
  float* dst;
  int n, rows, sstride, dstride;
  unsigned mask;
  uint32_t want;
};

__device__ __forceinline__ Seg seg1(const uint64_t* src, float* dst, int n, uint32_t want) {
  return Seg{src, dst, n, 1, n, n, 1u, want};
}

// Every phase thread polls its share of the region, kPollBatch words at a
// time (word f = tid + k * kPT of the batch), until each tag equals
// `want`, storing the values to shared memory; a word is re-read only while
// its tag is stale. Bounded: past sh.wait_ns, or when another CTA has failed,
// the CTA is marked failed (the caller checks after its next barrier). With
// `acquire`, a fence after the last observation orders this thread's later
// loads after the writers' release fences.
// Paired form of the poll: rows of even length and stride starting on a
// 16-byte boundary are read two words per load, PB pairs per thread per
// round, so a 1536-word region takes one round trip.
template <int PB>
__device__ __forceinline__ bool poll_pairs(const Seg& s, FlowShared& sh, int* status) {
  const int tid = threadIdx.x;
  const int np = s.n >> 1;
  const int total = s.rows * np;
  const unsigned long long t0 = now_ns();
  for (int base = 0; base < total; base += kPT * PB) {
    uint32_t so[PB], dof[PB];
    unsigned pend = 0;  // bits 2k and 2k + 1: the two words of pair k
#pragma unroll
    for (int k = 0; k < PB; k++) {
      const int f = base + tid + k * kPT;
      so[k] = 0;
      dof[k] = 0;
      if (f < total) {
        const int r = f / np, c = f - r * np;
        if ((s.mask >> r) & 1u) {
          so[k] = (uint32_t)(r * s.sstride + 2 * c);
          dof[k] = (uint32_t)(r * s.dstride + 2 * c);
          pend |= 3u << (2 * k);
        }
      }
    }
    unsigned spins = 0;
    while (pend) {
      uint64_t w[2 * PB];
#pragma unroll
      for (int k = 0; k < PB; k++)
        if ((pend >> (2 * k)) & 3u) ld_word2(s.src + so[k], w[2 * k], w[2 * k + 1]);
#pragma unroll
      for (int k = 0; k < PB; k++) {
#pragma unroll
        for (int e = 0; e < 2; e++) {
          const unsigned bit = 1u << (2 * k + e);
          if ((pend & bit) && (uint32_t)(w[2 * k + e] >> 32) == s.want) {
            s.dst[dof[k] + e] = __uint_as_float((uint32_t)w[2 * k + e]);
            pend &= ~bit;
          }
        }
      }
      if (pend) {
        const unsigned long long el = now_ns() - t0;
        if ((++spins & 31u) == 0 && (failed(sh) || status_now(status) != kStOk)) {
          flag_fail(sh, status, kStOk);
          return false;
        }
        if (el > sh.wait_ns) {
          flag_fail(sh, status, kStTimeout);
          return false;
        }
        poll_backoff(el);
      }
    }
  }
  return true;
}

template <int PB = kPollBatch>
__device__ __forceinline__ void poll(const Seg& s, bool acquire, FlowShared& sh, int* status);

// One out-of-line copy of the poll for every stage (instead of one inlined
// copy per call site): the token loop's code then fits the instruction
// caches. Scalar arguments keep the region out of local memory.
template <int PB>
__device__ __noinline__ void poll_call(const uint64_t* src, float* dst, int n, int rows, int sstride, int dstride,
                                       unsigned mask, uint32_t want, int acquire, FlowShared* sh, int* status) {
  poll<PB>(Seg{src, dst, n, rows, sstride, dstride, mask, want}, acquire != 0, *sh, status);
}

template <int PB>
__device__ __forceinline__ void poll(const Seg& s, bool acquire, FlowShared& sh, int* status) {
  if (((s.n | s.sstride) & 1) == 0 && (reinterpret_cast<uintptr_t>(s.src) & 15) == 0) {
    poll_pairs<(PB + 1) / 2 < 4 ? 4 : (PB + 1) / 2>(s, sh, status);
    if (acquire) fence_acquire_gpu();
    return;
  }
  const int tid = threadIdx.x;
  const int total = s.rows * s.n;
  const unsigned long long t0 = now_ns();
  bool ok = true;
  for (int base = 0; ok && base < total; base += kPT * PB) {
    uint32_t so[PB], dof[PB];
    unsigned pend = 0;
#pragma unroll
    for (int k = 0; k < PB; k++) {
      const int f = base + tid + k * kPT;
      so[k] = 0;
      dof[k] = 0;
      if (f < total) {
        const int r = f / s.n, c = f - r * s.n;
        if ((s.mask >> r) & 1u) {
          so[k] = (uint32_t)(r * s.sstride + c);
          dof[k] = (uint32_t)(r * s.dstride + c);
          pend |= 1u << k;
        }
      }
    }
    unsigned spins = 0;
    while (pend) {
      uint64_t w[PB];
#pragma unroll
      for (int k = 0; k < PB; k++)
        if ((pend >> k) & 1u) w[k] = ld_word(s.src + so[k]);
#pragma unroll
      for (int k = 0; k < PB; k++) {
        if (((pend >> k) & 1u) && (uint32_t)(w[k] >> 32) == s.want) {
          s.dst[dof[k]] = __uint_as_float((uint32_t)w[k]);
          pend &= ~(1u << k);
        }
      }
      if (pend) {
        const unsigned long long el = now_ns() - t0;
        if ((++spins & 31u) == 0 && (failed(sh) || status_now(status) != kStOk)) {
          flag_fail(sh, status, kStOk);
          ok = false;
          break;
        }
        if (el > sh.wait_ns) {
          flag_fail(sh, status, kStTimeout);
          ok = false;
          break;
        }
        poll_backoff(el);
      }
    }
  }
  if (acquire) fence_acquire_gpu();
}

// ------------------------------------------------------------ weight ring
struct Ring {
  unsigned char* base;
  int slots, slot_bytes;
  uint64_t* full;
  uint64_t* empty;
  int p;  // phase threads: next piece to take; producer: next piece to issue
};

// Waits (bounded) for the next piece; returns its shared-memory address.
__device__ __forceinline__ const unsigned char* ring_wait(Ring& rg, FlowShared& sh, int* status) {
  const int slot = rg.p % rg.slots;
  const unsigned par = (unsigned)(rg.p / rg.slots) & 1u;
  if (!mbar_try_wait(&rg.full[slot], par)) {
    const unsigned long long t0 = now_ns();
    unsigned spins = 0;
    while (!mbar_try_wait(&rg.full[slot], par)) {
      if ((++spins & 63u) == 0) {
        if (failed(sh) || *(volatile int*)&sh.pfail) {
          flag_fail(sh, status, kStOk);
          break;
        }
        if (now_ns() - t0 > sh.wait_ns) {
          flag_fail(sh, status, kStTimeout);
          break;
        }
      }
    }
  }
  return rg.base + (size_t)slot * rg.slot_bytes;
}

// Each phase warp hands the piece back once it has read its rows.
__device__ __forceinline__ void ring_release(Ring& rg) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&rg.empty[rg.p % rg.slots]);
  rg.p++;
}

// This CTA's rows of one matrix: [row0, row0 + nrows), rb bytes each, cut
// into ring pieces of `per` rows (even for the pair-interleaved matrices).
struct Slice {
  const unsigned char* src;
  int row0, nrows, rb, per;
};

// kind: 0 QKV, 1 O, 2 gate/up, 3 down, 4 lm_head.
__device__ Slice slice_of(const DModel& m, const DLayer* ly, int nblk, int kind, int l, int cta, int ncta,
                          int slot_bytes) {
  const int ws = m.bf16 ? 2 : 4;
  Slice s;
  int u0, u1;
  if (kind == 0) {
    cta_range(m.QKVR / 2, cta, ncta, u0, u1);
    s.row0 = 2 * u0;
    s.nrows = 2 * (u1 - u0);
    s.rb = m.H * ws;
    s.src = static_cast<const unsigned char*>(ly[l].wqkv);
  } else if (kind == 1) {
    cta_range(m.H, cta, ncta, u0, u1);
    s.row0 = u0;
    s.nrows = u1 - u0;
    s.rb = m.QD * ws;
    s.src = static_cast<const unsigned char*>(ly[l].wo);
  } else if (kind == 2) {
    cta_range(m.FF, cta, ncta, u0, u1);
    s.row0 = 2 * u0;
    s.nrows = 2 * (u1 - u0);
    s.rb = m.H * ws;
    s.src = static_cast<const unsigned char*>(ly[l].wgu);
  } else if (kind == 3) {
    cta_range(m.H, cta, ncta, u0, u1);
    s.row0 = u0;
    s.nrows = u1 - u0;
    s.rb = m.FF * ws;
    s.src = static_cast<const unsigned char*>(ly[l].wdown);
  } else {
    cta_range(nblk, cta, ncta, u0, u1);
    s.row0 = u0 * kSBlk;
    s.nrows = max(0, min(u1 * kSBlk, m.V) - s.row0);
    s.rb = m.H * ws;
    s.src = static_cast<const unsigned char*>(m.head);
  }
  s.src += (size_t)s.row0 * s.rb;
  s.per = slot_bytes / s.rb;
  if (kind == 0 || kind == 2) s.per &= ~1;
  if (s.per < 1) s.nrows = 0;  // never reached: flow_plan sizes slots for two rows
  return s;
}

// Producer (one thread): this CTA's pieces in consumption order, step by
// step, until the run ends or the phase threads stop; then waits until every
// copy it issued has landed.
__device__ void produce(const DModel& m, const DLayer* ly, int nblk, Ring& rg, FlowShared& sh, int nsteps, int cta,
                        int ncta, int* status) {
  bool stopped = false;
  const uint64_t pol_layer = policy_evict_first(), pol_head = policy_evict_last();
  for (int s = 0; s < nsteps && !stopped; s++) {
    for (int l = 0; l <= m.L && !stopped; l++) {
      const int nk = l < m.L ? 4 : 1;
      for (int k = 0; k < nk && !stopped; k++) {
        const Slice sl = slice_of(m, ly, nblk, l < m.L ? k : 4, l, cta, ncta, rg.slot_bytes);
        for (int done = 0; done < sl.nrows && !stopped;) {
          const int n = min(sl.per, sl.nrows - done);
          const int slot = rg.p % rg.slots;
          if (rg.p >= rg.slots) {
            const unsigned par = (unsigned)(rg.p / rg.slots - 1) & 1u;
            const unsigned long long t0 = now_ns();
            unsigned spins = 0;
            while (!mbar_try_wait(&rg.empty[slot], par)) {
              if (*(volatile int*)&sh.stop) {
                stopped = true;
                break;
              }
              if ((++spins & 63u) == 0 && now_ns() - t0 > kProducerWaitNs) {
                producer_fail(sh, status);
                stopped = true;
                break;
              }
            }
            if (stopped) break;
          }
          const unsigned bytes = (unsigned)(n * sl.rb);
          mbar_expect_tx(&rg.full[slot], bytes);
          bulk_g2s_hint(rg.base + (size_t)slot * rg.slot_bytes, sl.src + (size_t)done * sl.rb, bytes, &rg.full[slot],
                        l < m.L ? pol_layer : pol_head);
          rg.p++;
          done += n;
        }
      }
    }
  }
  // The last piece issued into each slot is the only one that can still be
  // in flight there.
  for (int q = max(0, rg.p - rg.slots); q < rg.p; q++) {
    const int slot = q % rg.slots;
    const unsigned par = (unsigned)(q / rg.slots) & 1u;
    const unsigned long long t0 = now_ns();
    unsigned spins = 0;
    while (!mbar_try_wait(&rg.full[slot], par)) {
      if ((++spins & 63u) == 0 && now_ns() - t0 > kProducerWaitNs) {
        producer_fail(sh, status);
        break;
      }
    }
  }
}

// Canonical warp dot product (the rule of warp_dot) with the weight rows in
// shared memory; with NORM the inputs are first RMS-normalised element by
// element, n = (x * inv[g]) * w (the rounding of stage_norm).
template <bool BF16, bool NORM, int NR, int G>
__device__ __forceinline__ void warp_dot_smem(const void* const (&rows)[NR], int K, const float* xs, int xstride,
                                              const float* nw, const float (&inv)[G], float (&acc)[NR][G]) {
  constexpr int E = BF16 ? 8 : 4;
  const int lane = threadIdx.x & 31;
  const int nch = K / E;
#pragma unroll
  for (int r = 0; r < NR; r++)
#pragma unroll
    for (int g = 0; g < G; g++) acc[r][g] = 0.0f;
#pragma unroll 4
  for (int j = lane; j < nch; j += 32) {
    float w[NR][E];
#pragma unroll
    for (int r = 0; r < NR; r++) {
      if constexpr (BF16) {
        const uint4 t = reinterpret_cast<const uint4*>(rows[r])[j];
        w[r][0] = bf16_lo(t.x);
        w[r][1] = bf16_hi(t.x);
        w[r][2] = bf16_lo(t.y);
        w[r][3] = bf16_hi(t.y);
        w[r][4] = bf16_lo(t.z);
        w[r][5] = bf16_hi(t.z);
        w[r][6] = bf16_lo(t.w);
        w[r][7] = bf16_hi(t.w);
      } else {
        const float4 t = reinterpret_cast<const float4*>(rows[r])[j];
        w[r][0] = t.x;
        w[r][1] = t.y;
        w[r][2] = t.z;
        w[r][3] = t.w;
      }
    }
    float wn[E];
    if (NORM) {
#pragma unroll
      for (int q = 0; q < E / 4; q++) {
        const float4 t = *reinterpret_cast<const float4*>(nw + j * E + 4 * q);
        wn[4 * q] = t.x;
        wn[4 * q + 1] = t.y;
        wn[4 * q + 2] = t.z;
        wn[4 * q + 3] = t.w;
      }
    }
#pragma unroll
    for (int g = 0; g < G; g++) {
      float xv[E];
#pragma unroll
      for (int q = 0; q < E / 4; q++) {
        const float4 t = *reinterpret_cast<const float4*>(xs + (size_t)g * xstride + j * E + 4 * q);
        xv[4 * q] = t.x;
        xv[4 * q + 1] = t.y;
        xv[4 * q + 2] = t.z;
        xv[4 * q + 3] = t.w;
      }
      if (NORM) {
#pragma unroll
        for (int e = 0; e < E; e++) xv[e] = __fmul_rn(__fmul_rn(xv[e], inv[g]), wn[e]);
      }
#pragma unroll
      for (int r = 0; r < NR; r++)
#pragma unroll
        for (int e = 0; e < E; e++) acc[r][g] = fmaf(w[r][e], xv[e], acc[r][g]);
    }
  }
#pragma unroll
  for (int r = 0; r < NR; r++)
#pragma unroll
    for (int g = 0; g < G; g++) acc[r][g] = warp_sum_butterfly(acc[r][g]);
}

// ------------------------------------------------------------ phase threads
template <bool BF16, int G>
struct Flow {
  const DModel& m;
  const DBatch& bt;
  const FlowBufs& fb;
  const FlowGeo& geo;
  FlowShared& sh;
  Ring& rg;
  int cta, ncta, nblk, KS;
  float* stage;  // staging area (geo.stage_f floats)
  float* ol;     // [G][ol_f] this CTA's logits
  float* ownx;   // [G][ox_f] this CTA's residual rows
  float* rope;   // [G][2 HALF]
  float* nw;     // [H] norm weights of the current stage
  const DLayer* ly;  // [L] layer table (shared memory)
  int k0, k1;    // this CTA's logits blocks
  int r0, r1;    // this CTA's residual rows
  bool has_kv;   // this CTA's QKV rows include K/V rows (it appends to the cache)
  int cur_s = -1, cur_sid = 0;  // the stage being traced (instrumentation)

  __device__ uint32_t tag(int s, int id) const { return fb.epoch + (uint32_t)((s + 1) * KS + id); }

  // Trace stamps of step bt.trace_step (instrumentation; off when bt.trace
  // is null): stage entry and inputs received by thread 0, done per warp.
  __device__ void tr_at(int s, int sid, int slot) const {
    if (bt.trace && s == bt.trace_step && sid < KS)
      bt.trace[((size_t)cta * KS + sid) * kTraceSlots + slot] = now_ns();
  }
  __device__ void tr_entry(int s, int sid) {
    cur_s = s;
    cur_sid = sid;
    if (threadIdx.x == 0) tr_at(s, sid, 0);
  }
  // A sub-stage mark of the current stage by warp 0.
  __device__ void tr_mark(int slot) const {
    if (threadIdx.x == 0) tr_at(cur_s, cur_sid, slot);
  }
  __device__ void tr_recv(int s, int sid) const {
    if (threadIdx.x == 0) tr_at(s, sid, 1);
  }
  __device__ void tr_done(int s, int sid) const {
    if ((threadIdx.x & 31) == 0) tr_at(s, sid, 2 + (threadIdx.x >> 5));
  }
  __device__ bool fail() const { return failed(sh); }
  __device__ unsigned act_mask() const {
    unsigned mk = 0;
#pragma unroll
    for (int g = 0; g < G; g++)
      if (sh.act[g]) mk |= 1u << g;
    return mk;
  }
  template <int PB = kPollBatch>
  __device__ void do_poll(const Seg& s, bool acquire) {
    poll_call<PB>(s.src, s.dst, s.n, s.rows, s.sstride, s.dstride, s.mask, s.want, acquire ? 1 : 0, &sh, bt.status);
  }

  // Norm weights of a stage: copied global -> shared with cp.async before
  // the poll (no registers held, the copy overlaps the wait); norm_ready()
  // after the poll, followed by a phase barrier, makes them visible.
  __device__ void load_norm(const float* w) {
    for (int c = threadIdx.x; c < m.H / 4; c += kPT) cp_async16(nw + 4 * c, w + 4 * c);
    cp_async_commit();
  }
  __device__ static void norm_ready() { cp_async_wait_all(); }

  // 1 / sqrt(ss / H + eps) for slot g's staged x, by one warp (every lane
  // gets it); ss follows the canonical dot rule (lane-strided float4 chunks,
  // fmaf in element order, xor butterfly), as stage_norm does.
  __device__ float inv_rms(const float* xr, int stride, int g) const {
    const int lane = threadIdx.x & 31;
    const float4* x4 = reinterpret_cast<const float4*>(xr + (size_t)g * stride);
    float acc = 0.0f;
    for (int j = lane; j < m.H / 4; j += 32) {
      const float4 t = x4[j];
      acc = fmaf(t.x, t.x, acc);
      acc = fmaf(t.y, t.y, acc);
      acc = fmaf(t.z, t.z, acc);
      acc = fmaf(t.w, t.w, acc);
    }
    acc = warp_sum_butterfly(acc);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)m.H), m.eps)));
  }

  __device__ static void csync_() { DEFER_CTA_SYNC(); }

  // The epilogue of rows `row` (and `row + 1` when has1) of a projection.
  __device__ void epi(int kind, int l, uint32_t tg, int row, const float* a0, bool has1, const float* a1) {
    if (kind == kEpiResid) {
      resid(row, a0, tg);
      if (has1) resid(row + 1, a1, tg);
      return;
    }
    if (kind == kEpiHead) {

      const int lane = threadIdx.x & 31;
#pragma unroll
      for (int g = 0; g < G; g++) {
        if (lane != g) continue;
        ol[(size_t)g * geo.ol_f + (row - k0 * kSBlk)] = a0[g];
        if (has1) ol[(size_t)g * geo.ol_f + (row + 1 - k0 * kSBlk)] = a1[g];
      }
      return;
    }
    if (kind == kEpiGateUp) {

      const int j = row >> 1;
      const int lane = threadIdx.x & 31;
#pragma unroll
      for (int g = 0; g < G; g++) {
        if (lane != g || !sh.act[g]) continue;
        const float gate = a0[g], up = a1[g];
        float act;
        if (m.gelu != 0) {
          const float C = 0.7978846f;
          const float x3 = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, gate), gate), gate);
          act = __fmul_rn(__fmul_rn(0.5f, gate), __fadd_rn(1.0f, tanhf(__fmul_rn(C, __fadd_rn(gate, x3)))));
        } else {
          act = __fdiv_rn(gate, __fadd_rn(1.0f, expf(-gate)));
        }
        st_f(fb.gt + (size_t)g * m.FF + j, __fmul_rn(act, up), tg);
      }
      return;
    }
    // kEpiQkv
    const DLayer& Ly = ly[l];
    const int HD = m.HD, HALF = m.HALF, Gh = m.NH / m.NKV;
    const int qh = m.QD / 2, kh = m.KVD / 2, grp = (Gh + 2) * HD;
    const int qkvd = m.QD + 2 * m.KVD;

      const int u = row >> 1;
      int sect, h, i;
      if (u < qh) {
        sect = 0;
        h = u / HALF;
        i = u % HALF;
      } else if (u < qh + kh) {
        sect = 1;
        h = (u - qh) / HALF;
        i = (u - qh) % HALF;
      } else {
        sect = 2;
        h = (u - qh - kh) / HALF;
        i = (u - qh - kh) % HALF;
      }
      const int lane = threadIdx.x & 31;
#pragma unroll
      for (int g = 0; g < G; g++) {
        if (lane != g || !sh.act[g]) continue;
        float a = a0[g], c = a1[g];
        if (Ly.bqkv) {
          a = __fadd_rn(a, Ly.bqkv[2 * u]);
          c = __fadd_rn(c, Ly.bqkv[2 * u + 1]);
        }
        if (sect < 2) {
          const float cs = rope[(size_t)g * geo.rope_f + i];
          const float sn = rope[(size_t)g * geo.rope_f + HALF + i];
          const float a2 = __fsub_rn(__fmul_rn(a, cs), __fmul_rn(c, sn));
          const float c2 = __fadd_rn(__fmul_rn(c, cs), __fmul_rn(a, sn));
          a = a2;
          c = c2;
        }
        uint64_t* qrow = fb.qt + (size_t)g * qkvd;
        if (sect == 0) {
          uint64_t* d = qrow + (size_t)(h / Gh) * grp + (h % Gh) * HD;
          st_f(d + i, a, tg);
          st_f(d + i + HALF, c, tg);
        } else {
          const DSession& S = sh.sess[g];
          float* dst = (sect == 1 ? S.kc : S.vc) + (((size_t)l * m.NKV + h) * S.cap + sh.pos[g]) * HD;
          dst[i] = a;
          dst[i + HALF] = c;
          uint64_t* d = qrow + (size_t)h * grp + (Gh + sect - 1) * HD;
          st_f(d + i, a, tg);
          st_f(d + i + HALF, c, tg);
        }
      }
  }

  // This CTA's rows of a slice from the ring against the staged inputs
  // xs[g * xstride + k] (k < K), warp by warp with no CTA barrier: each warp
  // takes row pairs of every piece and hands their sums to
  // epi(row, acc_row[G], has_second_row, acc_second[G]). With NORM the inputs
  // are RMS-normalised on the fly, n = (x * inv) * w with the norm weights
  // staged in nw (the rounding of stage_norm); each warp computes inv.
  // NR rows (2 or 4) per warp pass; the epilogue still sees row pairs.
  // Epilogue kinds of gemv (one projection loop per normalisation mode,
  // the epilogue chosen at run time, so the loop's code exists twice, not
  // once per stage).
  enum { kEpiQkv = 0, kEpiResid = 1, kEpiGateUp = 2, kEpiHead = 3 };

  template <bool NORM, int NR = 2>
  __device__ void gemv(const Slice& sl, const float* xs, int xstride, int K, int kind, int l, uint32_t tg) {
    const int warp = threadIdx.x >> 5;
    float inv[G];
    if (NORM && G == 1) {
      inv[0] = sh.act[0] ? inv_rms(xs, xstride, 0) : 0.0f;  // every warp, no barrier
      tr_mark(10);
    } else if (NORM) {
      // slot g's statistic once for the CTA, by warp g mod 7 (same rule)
      for (int g = warp; g < G; g += kPW) {
        if (!sh.act[g]) continue;
        const float v = inv_rms(xs, xstride, g);
        if ((threadIdx.x & 31) == 0) sh.inv[g] = v;
      }
      csync_();
#pragma unroll
      for (int g = 0; g < G; g++) inv[g] = sh.act[g] ? sh.inv[g] : 0.0f;
    } else {
#pragma unroll
      for (int g = 0; g < G; g++) inv[g] = 0.0f;
    }
    for (int done = 0; done < sl.nrows;) {
      const int n = min(sl.per, sl.nrows - done);
      const unsigned char* base = ring_wait(rg, sh, bt.status);
      if (done == 0) tr_mark(11);
      for (int pr = warp; NR * pr < n; pr += kPW) {
        const int i0 = NR * pr;
        const void* rows[NR];
#pragma unroll
        for (int r = 0; r < NR; r++) rows[r] = base + (size_t)min(i0 + r, n - 1) * sl.rb;
        float acc[NR][G];
        warp_dot_smem<BF16, NORM, NR, G>(rows, K, xs, xstride, nw, inv, acc);
#pragma unroll
        for (int q = 0; q < NR / 2; q++)
          if (i0 + 2 * q < n) epi(kind, l, tg, sl.row0 + done + i0 + 2 * q, acc[2 * q], i0 + 2 * q + 1 < n, acc[2 * q + 1]);
      }
      ring_release(rg);
      done += n;
    }
  }

  // x[r] += a for the slots (O and down projections), owner rows only.
  __device__ void resid(int r, const float* a, uint32_t tg) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int g = 0; g < G; g++) {
      if (lane != g || !sh.act[g]) continue;
      float* xo = ownx + (size_t)g * geo.ox_f + (r - r0);
      const float xn = __fadd_rn(*xo, a[g]);
      *xo = xn;
      st_f(fb.xt + (size_t)g * fb.xw + r, xn, tg);
    }
  }

  // ------------------------------------------------- distributed sampler
  // The exact sampler (phases.cuh) with its row passes spread over every
  // CTA: each CTA computes the records (predicted binade and increments)
  // of its own logits rows, which it holds in shared memory since its head
  // stage, and publishes them as tagged words; the slot's owner CTA polls
  // all records and walks them. Record of a row: word 0 = d0, word 1 =
  // binade code (e + 128; 254 all-zero row, 255 no prediction) | (d1 - d0 +
  // 32768) << 8.

  // Sum over the CTA's phase threads (any order; every thread gets it).
  __device__ float cta_sum_any(float v) {
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if ((threadIdx.x & 31) == 0) sh.ws[threadIdx.x >> 5][0] = v;
    csync_();
    float t = 0.0f;
    for (int w = 0; w < kPW; w++) t += sh.ws[w][0];
    csync_();
    return t;
  }

  // Records of this CTA's rows of slot g's logits for the pass `cdf` (p = e
  // * inv) or the sum of e, published with tag tg. Whole CTA.
  __device__ void sampler_records(int g, float M, float inv, bool cdf, uint32_t tg) {
    const float* rm = reinterpret_cast<const float*>(fb.esum) + (size_t)g * 2 * nblk;
    const float* rz = rm + nblk;
    const float scale = cdf ? inv : 1.0f;
    // approximate running sum before this CTA's first row (any order)
    float pre = 0.0f;
    for (int r = threadIdx.x; r < k0; r += kPT) {
      const float z = ld_f(rz + r);
      pre += z > 0.0f ? z * expf(ld_f(rm + r) - M) * scale : 0.0f;
    }
    pre = cta_sum_any(pre);
    if (threadIdx.x < 32)
      records_rows(ol + (size_t)g * geo.ol_f, k0, k1, m.V, sh.sess[g].temperature, M, inv, cdf ? 1 : 0, rm, rz, pre,
                   (cdf ? fb.crec : fb.zrec) + (size_t)g * nblk * 2, stage, tg);
    csync_();
  }

  // The owner's walk over every CTA's records of slot b (tag tg): the sum of
  // e (cdf false) or the CDF search for r. Whole CTA; false on failure.
  __device__ bool sampler_walk(int b, float M, float inv, bool cdf, float r, uint32_t tg, float* total, int* hit,
                               float* prev, float* at) {
    do_poll(seg1((cdf ? fb.crec : fb.zrec) + (size_t)b * nblk * 2, stage, 2 * nblk, tg), false);
    csync_();
    if (fail()) return false;
    unsigned long long* mk = (bt.trace && cur_s == bt.trace_step && cur_sid == 0)
                                 ? bt.trace + (size_t)cta * KS * kTraceSlots + (cdf ? 19 : 16)
                                 : nullptr;
    if (mk && threadIdx.x == 0) mk[0] = now_ns();
    *total = walk_records(stage, m.V, bt.logits + (size_t)b * m.V, sh.sess[b].temperature, M, inv, cdf ? 1 : 0, r, hit,
                          prev, at, mk ? mk + 1 : nullptr);
    return true;
  }

  // ------------------------------------------------------------ select
  // Slot state update and token choice of step s for the slots this CTA
  // owns (ph_select), then the slot's step header: x = embedding row, step
  // info, RoPE rows. Returns false on failure.
  __device__ bool select(int s, unsigned first) {
    const int tid = threadIdx.x;
    const uint32_t tg = tag(s, 0);
    tr_entry(s, 0);
    // Fault drill (bt.stall): CTA 0 withholds the step header of step 0, so
    // every other CTA's first poll runs into its bounded wait.
    const bool withhold = bt.stall && s == 0 && cta == 0;
    // Slots that sample at this step, known to every CTA: the previous
    // step's header says so (or, at a run's first step, its programs).
    unsigned smask = s == 0 ? first : 0u;
    if (s > 0)
      for (int g = 0; g < bt.B; g++)
        if (sh.samp[g]) smask |= 1u << g;
    if (smask) {
      tr_mark(10);
      const uint32_t tz = tag(s, sid_s1(m.L)), tc = tag(s, sid_s2(m.L));
      // every CTA: M (the largest of the CTAs' maxima of s; each CTA
      // released its logits and row statistics before its maximum) and the
      // records of its rows in the sum of e
      for (int g = 0; g < bt.B; g++) {
        if (!((smask >> g) & 1u)) continue;
        do_poll(Seg{fb.csm + (size_t)g * fb.cta_cap, stage, ncta, 1, fb.cta_cap, ncta, 1u,
                    tag(s - 1, sid_head(m.L))},
                true);
        csync_();
        if (fail()) return false;
        float mx = -INFINITY;
        for (int j = tid; j < ncta; j += kPT) mx = fmaxf(mx, stage[j]);
        mx = cta_max(mx);
        if (tid == 0) sh.M[g] = mx;
        sampler_records(g, mx, 0.0f, false, tz);
      }
      tr_mark(12);
      // owners: the exact sum, and 1 / sum for every CTA
      for (int b = cta; b < bt.B; b += ncta) {
        if (!((smask >> b) & 1u)) continue;
        float Z, pv, at;
        int hit;
        if (!sampler_walk(b, sh.M[b], 0.0f, false, 0.0f, tz, &Z, &hit, &pv, &at)) return false;
        const float inv = (Z > 0.0f && isfinite(Z)) ? __fdiv_rn(1.0f, Z) : 0.0f;
        if (tid == 0) {
          sh.Z[b] = Z;
          sh.inv[b] = inv;
          st_f(fb.invw + b, inv, tc);
        }
        csync_();
      }
      tr_mark(13);
      // every CTA: the records of its rows in the CDF of p = e * (1 / sum)
      for (int g = 0; g < bt.B; g++) {
        if (!((smask >> g) & 1u)) continue;
        do_poll(seg1(fb.invw + g, stage, 1, tc), false);
        csync_();
        if (fail()) return false;
        const float inv = stage[0];
        csync_();
        sampler_records(g, sh.M[g], inv, true, tc);
      }
      tr_mark(14);
    }
    for (int b = cta; b < bt.B; b += ncta) {
      DSlotState* st = sh.st + b;
      const DSession& S = sh.sess[b];
      if (tid == 0) {
        if (st->was_active) {
          st->pos += 1;
          st->step += 1;
        }
        st->was_active = 0;
        st->active = 0;
        if (st->step >= S.n_total) st->done = 1;
        sh.go = !st->done;
        sh.step = st->step;
        sh.tok = 0xFFFFFFFFu;
        sh.sampn = 0;
      }
      csync_();
      if (sh.go) {
        const int si = sh.step;
        uint32_t tok;
        if (si < S.n_prompt) {
          tok = S.tokens[si];
        } else {
          const int k = si - S.n_prompt;
          const float T = S.temperature;
          float margin = 0.0f;
          uint32_t smp;
          if (T != 0.0f && ((smask >> b) & 1u) && sh.Z[b] > 0.0f && isfinite(sh.Z[b])) {
            // the CDF walk over every CTA's records
            const float inv = sh.inv[b];
            const float r = (float)(S.words[k] >> 8) * (1.0f / 16777216.0f);
            float total, pv, at;
            int hit;
            if (!sampler_walk(b, sh.M[b], inv, true, r, tag(s, sid_s2(m.L)), &total, &hit, &pv, &at)) return false;
            if (hit >= 0) {
              smp = (uint32_t)hit;
              margin = fminf(__fsub_rn(r, pv), __fsub_rn(at, r));
            } else {  // r past the last CDF value: the last index with p > 0
              const SampleVals vp{bt.logits + (size_t)b * m.V, T, sh.M[b], inv, true};
              const int last = last_positive(vp, m.V);
              smp = (uint32_t)(last < 0 ? 0 : last);
              margin = __fsub_rn(r, total);
            }
            tr_mark(15);
            tr_mark(11);
          } else if (T != 0.0f && !((smask >> b) & 1u)) {
            // (not announced by the previous header: the single-CTA sampler)
            // The previous step's logits are complete once every CTA's head
            // words are: each CTA released its logits stores before them.
            do_poll(Seg{fb.csm + (size_t)b * fb.cta_cap, stage, ncta, 1, fb.cta_cap, ncta, 1u,
                        tag(s - 1, sid_head(m.L))},
                    true);
            csync_();
            if (fail()) return false;
            // M = the largest of the CTAs' maxima of s
            float mx = -INFINITY;
            for (int j = tid; j < ncta; j += kPT) mx = fmaxf(mx, stage[j]);
            mx = cta_max(mx);
            tr_mark(10);
            const float* rm = reinterpret_cast<const float*>(fb.esum) + (size_t)b * 2 * nblk;
            unsigned long long* mk =
                (bt.trace && s == bt.trace_step) ? bt.trace + (size_t)cta * KS * kTraceSlots + 12 : nullptr;
            smp = sample_exact(bt.logits + (size_t)b * m.V, m.V, T, S.words[k], &margin, stage, true, mx, rm,
                               rm + nblk, mk);
            tr_mark(11);
          } else {
            // greedy, or a degenerate sum of e (the reference's one-hot argmax)
            if (T != 0.0f) margin = NAN;
            float* pr = stage;
            float* lm = stage + 2 * ncta;
            int* la = reinterpret_cast<int*>(lm + ncta);
            do_poll(seg1(fb.cl + (size_t)b * fb.cta_cap * 2, pr, 2 * ncta, tag(s - 1, sid_head(m.L))), false);
            csync_();
            if (fail()) return false;
            for (int j = tid; j < ncta; j += kPT) {
              lm[j] = pr[2 * j];
              la[j] = __float_as_int(pr[2 * j + 1]);
            }
            csync_();
            smp = argmax_from_blocks(lm, la, ncta, false);
          }
          if (S.verify) {
            tok = S.tokens[si];
            if (tid == 0 && smp != tok) {
              st->div_step = si;
              st->div_token = smp;
              st->done = 1;
            }
          } else {
            tok = smp;
            if (tid == 0) S.tokens[si] = smp;
          }
          if (tid == 0 && S.margins) S.margins[k] = margin;
        }
        if (tid == 0) {
          if (!st->done) {
            if (tok >= (uint32_t)m.V) {
              atomicCAS(bt.status, kStOk, kStBadToken);
              st->done = 1;
            } else if (st->pos >= m.max_seq || st->pos >= S.cap) {
              atomicCAS(bt.status, kStOk, kStContext);
              st->done = 1;
            } else {
              st->cur = tok;
              st->active = 1;
              st->was_active = 1;
              sh.tok = tok;
              if (!S.verify && si >= S.n_prompt) {
                for (int i = 0; i < S.n_stop; i++)
                  if ((i < kStopCache ? sh.stops[b][i] : S.stop[i]) == tok) st->done = 1;  // fed now, nothing after it
              }
              const int nxt = si + 1;
              sh.sampn = S.temperature != 0.0f && !st->done && nxt >= S.n_prompt && nxt < S.n_total;
            }
          }
        }
        csync_();
      }
      // Step header (written for every slot, active or not).
      const uint32_t t = sh.tok;
      const bool live = t != 0xFFFFFFFFu;
      const int pos = live ? st->pos : -1;
      uint64_t* xrow = fb.xt + (size_t)b * fb.xw;
      // x = embedding row (kNormRegs words per thread cover H), RoPE rows:
      // every load in flight before the stores
      float ev[kNormRegs];
#pragma unroll
      for (int k = 0; k < kNormRegs; k++) {
        const int i = tid + k * kPT;
        ev[k] = 0.0f;
        if (live && i < m.H) {
          if (BF16)
            ev[k] = __uint_as_float((uint32_t)(reinterpret_cast<const uint16_t*>(m.embed) + (size_t)t * m.H)[i] << 16);
          else
            ev[k] = (reinterpret_cast<const float*>(m.embed) + (size_t)t * m.H)[i];
        }
      }
      float rc = 0.0f, rs = 0.0f;
      if (live && tid < m.HALF) {
        rc = m.rope_cos[(size_t)pos * m.HALF + tid];
        rs = m.rope_sin[(size_t)pos * m.HALF + tid];
      }
      if (!withhold) {
#pragma unroll
        for (int k = 0; k < kNormRegs; k++) {
          const int i = tid + k * kPT;
          if (i < m.H) st_f(xrow + i, ev[k], tg);
        }
        if (tid < m.HALF) {
          st_f(xrow + m.H + 2 + tid, rc, tg);
          st_f(xrow + m.H + 2 + m.HALF + tid, rs, tg);
        }
        if (tid == 0) {
          st_word(xrow + m.H, (uint32_t)pos, tg);
          st_word(xrow + m.H + 1, (live ? (t & 0x7FFFFFFFu) : 0u) | (sh.sampn ? 0x80000000u : 0u), tg);
        }
      }
      csync_();
    }
    tr_done(s, 0);
    return true;
  }

  // --------------------------------------------------------------- QKV
  // Returns false when the run ends (no active slot) or on failure.
  __device__ bool qkv(int s, int l) {
    tr_entry(s, sid_qkv(l));
    const Slice sl = slice_of(m, ly, nblk, 0, l, cta, ncta, geo.slot_bytes);
    const DLayer& Ly = ly[l];
    if (sl.nrows > 0) load_norm(Ly.attn_norm);
    const int H = m.H, xw = fb.xw;
    float* xr = stage;
    int xstride;
    csync_();  // the previous stage's warps are done with the staging area
    if (l == 0) {
      // the step header of every slot
      const unsigned all = (1u << bt.B) - 1u;
      const uint32_t tg = tag(s, 0);
      const int hn = H + 2 + 2 * m.HALF;  // header words written (the rest is padding)
      if (sl.nrows > 0) {
        do_poll(Seg{fb.xt, xr, hn, bt.B, xw, xw, all, tg}, false);
      } else {
        do_poll(Seg{fb.xt + H, xr + H, hn - H, bt.B, xw, xw, all, tg}, false);
        if (r1 > r0) do_poll(Seg{fb.xt + r0, xr + r0, r1 - r0, bt.B, xw, xw, all, tg}, false);
      }
      if (sl.nrows > 0) norm_ready();
      fence_acquire_gpu();  // as acquire_cache (the positions are known below)
      csync_();
      if (fail()) return false;
      tr_recv(s, sid_qkv(l));
      if (threadIdx.x < G) {
        const int g = threadIdx.x;
        int p = -1, smp = 0;
        if (g < bt.B) {
          p = __float_as_int(xr[(size_t)g * xw + H]);
          smp = (int)(__float_as_uint(xr[(size_t)g * xw + H + 1]) >> 31);
        }
        sh.act[g] = p >= 0;
        sh.pos[g] = p;
        sh.samp[g] = p >= 0 && smp;
      }
      for (int g = 0; g < bt.B; g++) {
        for (int i = threadIdx.x; i < 2 * m.HALF; i += kPT)
          rope[(size_t)g * geo.rope_f + i] = xr[(size_t)g * xw + H + 2 + i];
        for (int r = r0 + (int)threadIdx.x; r < r1; r += kPT)
          ownx[(size_t)g * geo.ox_f + (r - r0)] = xr[(size_t)g * xw + r];
      }
      csync_();
      if (!act_mask()) return false;
      prefetch_chunks(0);
      xstride = xw;
    } else {
      const unsigned act = act_mask();
      const uint32_t tg = tag(s, sid_dn(l - 1));
      if (sl.nrows > 0) {
        do_poll(Seg{fb.xt, xr, H, G, xw, H, act, tg}, false);
        norm_ready();
      } else if (r1 > r0) {
        do_poll(Seg{fb.xt + r0, xr + r0, r1 - r0, G, xw, H, act, tg}, false);
      }
      acquire_cache(l);
      csync_();
      if (fail()) return false;
      tr_recv(s, sid_qkv(l));
      // own residual rows (the O projection adds to them; read after barriers)
#pragma unroll
      for (int g = 0; g < G; g++) {
        if (!sh.act[g]) continue;
        for (int r = r0 + (int)threadIdx.x; r < r1; r += kPT)
          ownx[(size_t)g * geo.ox_f + (r - r0)] = xr[(size_t)g * H + r];
      }
      xstride = H;
    }
    if (sl.nrows == 0) {
      tr_done(s, sid_qkv(l));
      return true;
    }
    gemv<true>(sl, xr, xstride, H, kEpiQkv, l, tag(s, sid_qkv(l)));
    tr_done(s, sid_qkv(l));
    return true;
  }

  // Acquire: every CTA's KV-cache appends of earlier steps were released
  // before tagged words this thread has already observed (their O-stage
  // release, then gate/up words polled in the down stage), so after this
  // fence this layer's cached rows may be read. Placed after a poll, when
  // the thread's own recent stores (which the fence waits for) have drained.
  __device__ void acquire_cache(int l) {
    fence_acquire_gpu();
    prefetch_chunks(l);
  }

  // Moves the cached rows of this CTA's attention units of layer l into L2
  // (prefetches have no ordering effect).
  __device__ void prefetch_chunks(int l) {
    if (threadIdx.x != 0) return;
    const int maxc = bt.max_chunks, units = bt.B * m.NKV * maxc;
    for (int u = cta; u < units; u += ncta) {
      const int b = u / (m.NKV * maxc), rem = u % (m.NKV * maxc);
      const int kvh = rem / maxc, c = rem % maxc;
      if (!sh.act[b]) continue;
      const int pos = sh.pos[b], t0 = c * kAttnChunk;
      const int tc = min(kAttnChunk, pos - t0);
      if (tc <= 0) continue;
      const DSession& S = sh.sess[b];
      const size_t off = (((size_t)l * m.NKV + kvh) * S.cap + t0) * m.HD;
      prefetch_l2(S.kc + off, (size_t)tc * m.HD * sizeof(float));
      prefetch_l2(S.vc + off, (size_t)tc * m.HD * sizeof(float));
    }
  }

  // --------------------------------------------------------- attention
  // Units (slot, KV head, chunk of kAttnChunk positions) over the CTAs. The
  // cached rows (positions < pos) are loaded before the new q/k/v arrive:
  // every appending CTA released them at its O stage (release fence by all
  // its threads, then later tagged words that every CTA polls), and the
  // fence at the start of the QKV stage acquired them. A single-chunk unit
  // writes the output directly (the combine of one chunk is acc / l, bit for
  // bit); otherwise the partials of each (slot, query head) are combined, in
  // chunk order, by one CTA placed after the unit CTAs.
  __device__ bool attn(int s, int l) {
    tr_entry(s, sid_att(l));
    csync_();  // the QKV warps are done with the staging area
    const int Gh = m.NH / m.NKV, HD = m.HD, maxc = bt.max_chunks;
    const int grp = (Gh + 2) * HD;
    const int qkvd = m.QD + 2 * m.KVD;
    const int units = bt.B * m.NKV * maxc;
    const uint32_t tq = tag(s, sid_qkv(l)), tp = tag(s, sid_att(l));
    float* qs = stage;                        // [Gh][HD], then new k, new v
    float* kn = qs + Gh * HD;
    float* vn = kn + HD;
    float* sc = vn + HD;                      // [Gh][kAttnChunk]
    float* ks = sc + Gh * kAttnChunk;         // [kAttnChunk][HD + 4]
    float* vs = ks + kAttnChunk * (HD + 4);   // [kAttnChunk][HD]
    float* lsum = vs + kAttnChunk * HD;       // [Gh] chunk sums of e
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c4n = HD / 4;
    for (int u = cta; u < units; u += ncta) {
      const int b = u / (m.NKV * maxc);
      const int rem = u % (m.NKV * maxc);
      const int kvh = rem / maxc, c = rem % maxc;
      if (!sh.act[b]) continue;
      const int pos = sh.pos[b];
      const int nch = pos / kAttnChunk + 1;
      if (c >= nch) continue;
      const DSession& S = sh.sess[b];
      const int t0 = c * kAttnChunk;
      const int tn = min(kAttnChunk, pos + 1 - t0);  // rows of this chunk
      const int tc = min(tn, pos - t0);              // of which cached (t < pos)
      const size_t head_base = ((size_t)l * m.NKV + kvh) * S.cap;
      // Cached rows -> shared memory. The first batch's loads stay in flight
      // across the q/k/v poll; later batches (long heads) follow it.
      float4 kv[kKvBatch], vv[kKvBatch];
#pragma unroll
      for (int k = 0; k < kKvBatch; k++) {
        const int idx = tid + k * kPT;
        if (idx < tc * c4n) {
          const int tt = idx / c4n, c4 = idx - tt * c4n;
          kv[k] = ld_act(S.kc + (head_base + t0 + tt) * HD + 4 * c4);
          vv[k] = ld_act(S.vc + (head_base + t0 + tt) * HD + 4 * c4);
        }
      }
      do_poll(seg1(fb.qt + (size_t)b * qkvd + (size_t)kvh * grp, qs, grp, tq), false);
      for (int base = 0; base < tc * c4n; base += kKvBatch * kPT) {
        if (base > 0) {
#pragma unroll
          for (int k = 0; k < kKvBatch; k++) {
            const int idx = base + tid + k * kPT;
            if (idx < tc * c4n) {
              const int tt = idx / c4n, c4 = idx - tt * c4n;
              kv[k] = ld_act(S.kc + (head_base + t0 + tt) * HD + 4 * c4);
              vv[k] = ld_act(S.vc + (head_base + t0 + tt) * HD + 4 * c4);
            }
          }
        }
#pragma unroll
        for (int k = 0; k < kKvBatch; k++) {
          const int idx = base + tid + k * kPT;
          if (idx < tc * c4n) {
            const int tt = idx / c4n, c4 = idx - tt * c4n;
            *reinterpret_cast<float4*>(ks + (size_t)tt * (HD + 4) + 4 * c4) = kv[k];
            *reinterpret_cast<float4*>(vs + (size_t)tt * HD + 4 * c4) = vv[k];
          }
        }
      }
      if (u == cta) tr_recv(s, sid_att(l));
      csync_();
      if (fail()) return false;
      if (u == cta) tr_mark(10);
      // scores; the row of position pos (t == pos, last of the last chunk) is the new k
      for (int idx = tid; idx < Gh * kAttnChunk; idx += kPT) {
        const int h = idx / kAttnChunk, tt = idx - h * kAttnChunk;
        float sv = -INFINITY;
        const int t = t0 + tt;
        const bool masked = S.mask && t < pos && ((S.mask[t >> 5] >> (t & 31)) & 1u);
        if (tt < tn && !masked) {
          const float* kr = t == pos ? kn : ks + (size_t)tt * (HD + 4);
          const float* qr = qs + h * HD;
          float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll 4
          for (int d = 0; d < HD; d += 4) {
            const float4 k4 = *reinterpret_cast<const float4*>(kr + d);
            a0 = fmaf(qr[d], k4.x, a0);
            a1 = fmaf(qr[d + 1], k4.y, a1);
            a2 = fmaf(qr[d + 2], k4.z, a2);
            a3 = fmaf(qr[d + 3], k4.w, a3);
          }
          sv = __fmul_rn(__fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3)), m.scale);
        }
        sc[idx] = sv;
      }
      csync_();
      if (u == cta) tr_mark(11);
      const bool single = nch == 1;
      uint64_t* part = fb.pt + (((size_t)b * m.NH + (size_t)kvh * Gh) * maxc + c) * (HD + 2);
      const size_t hstride = (size_t)maxc * (HD + 2);
      for (int h = warp; h < Gh; h += kPW) {
        float* row = sc + h * kAttnChunk;
        const float v0 = row[lane], v1 = row[lane + 32];
        const float mx = warp_max(fmaxf(v0, v1));
        const float e0 = (v0 == -INFINITY) ? 0.0f : expf(__fsub_rn(v0, mx));
        const float e1 = (v1 == -INFINITY) ? 0.0f : expf(__fsub_rn(v1, mx));
        row[lane] = e0;
        row[lane + 32] = e1;
        const float ls = warp_sum_butterfly(__fadd_rn(e0, e1));
        if (lane == 0) {
          lsum[h] = ls;
          if (!single) {
            st_f(part + h * hstride, mx, tp);
            st_f(part + h * hstride + 1, ls, tp);
          }
        }
      }
      csync_();
      if (u == cta) tr_mark(12);
      const int tv = tn - (tc < tn ? 1 : 0);  // rows taken from vs (the new row, if any, comes last)
      for (int idx = tid; idx < Gh * HD; idx += kPT) {
        const int h = idx / HD, d = idx - h * HD;
        const float* e = sc + h * kAttnChunk;
        float acc = 0.0f;
#pragma unroll 8
        for (int tt = 0; tt < tv; tt++) acc = fmaf(e[tt], vs[(size_t)tt * HD + d], acc);
        if (tv < tn) acc = fmaf(e[tv], vn[d], acc);
        if (single)
          st_f(fb.at + (size_t)b * m.QD + (size_t)(kvh * Gh + h) * HD + d, __fdiv_rn(acc, lsum[h]), tp);
        else
          st_f(part + h * hstride + 2 + d, acc, tp);
      }
      csync_();
      if (u == cta) tr_mark(13);
    }
    tr_mark(14);
    // Combine per (slot, query head), chunks in order.
    for (int bh = 0; bh < bt.B * m.NH; bh++) {
      if ((units + bh) % ncta != cta) continue;
      const int b = bh / m.NH, h = bh % m.NH;
      if (!sh.act[b]) continue;
      const int nch = sh.pos[b] / kAttnChunk + 1;
      if (nch == 1) continue;  // written by its only unit
      const int row = nch * (HD + 2);
      const uint64_t* src = fb.pt + ((size_t)b * m.NH + h) * maxc * (HD + 2);
      do_poll<kCombineBatch>(seg1(src, stage, row, tp), false);
      csync_();
      if (fail()) return false;
      for (int d = tid; d < HD; d += kPT) {
        float M = -INFINITY;
        for (int cc = 0; cc < nch; cc++) M = fmaxf(M, stage[cc * (HD + 2)]);
        float L = 0.0f, O = 0.0f;
        for (int cc = 0; cc < nch; cc++) {
          const float* pc = stage + cc * (HD + 2);
          const float mc = pc[0], lc = pc[1], ac = pc[2 + d];
          const float w = (mc == -INFINITY) ? 0.0f : expf(__fsub_rn(mc, M));
          L = fmaf(w, lc, L);
          O = fmaf(w, ac, O);
        }
        st_f(fb.at + (size_t)b * m.QD + (size_t)h * HD + d, __fdiv_rn(O, L), tp);
      }
      csync_();
    }
    tr_mark(15);
    tr_done(s, sid_att(l));
    return true;
  }

  // --------------------------------------------------- O / gate-up / down
  __device__ bool oproj(int s, int l) {
    tr_entry(s, sid_o(l));
    const Slice sl = slice_of(m, ly, nblk, 1, l, cta, ncta, geo.slot_bytes);
    if (sl.nrows == 0) return true;
    csync_();
    do_poll(Seg{fb.at, stage, m.QD, G, m.QD, m.QD, act_mask(), tag(s, sid_att(l))}, false);
    csync_();
    if (fail()) return false;
    tr_recv(s, sid_o(l));
    const uint32_t tg = tag(s, sid_o(l));
    gemv<false>(sl, stage, m.QD, m.QD, kEpiResid, l, tg);
    tr_done(s, sid_o(l));
    return true;
  }

  __device__ bool gateup(int s, int l) {
    tr_entry(s, sid_gu(l));
    const Slice sl = slice_of(m, ly, nblk, 2, l, cta, ncta, geo.slot_bytes);
    if (sl.nrows == 0) return true;
    load_norm(ly[l].ffn_norm);
    csync_();
    do_poll(Seg{fb.xt, stage, m.H, G, fb.xw, m.H, act_mask(), tag(s, sid_o(l))}, false);
    norm_ready();
    csync_();
    if (fail()) return false;
    tr_recv(s, sid_gu(l));
    const uint32_t tg = tag(s, sid_gu(l));
    gemv<true>(sl, stage, m.H, m.H, kEpiGateUp, l, tg);  // the QKV loop's code: one copy stays in the i-cache
    tr_done(s, sid_gu(l));
    return true;
  }

  __device__ bool down(int s, int l) {
    tr_entry(s, sid_dn(l));
    // Release: after the stage barriers since this layer's QKV stage, a fence
    // in every thread of an appending CTA orders its cache appends before
    // its down-projection words, which every CTA polls in its next QKV
    // stage (and acquires). Here, before the poll, the fence's wait for the
    // thread's own stores overlaps the wait for the gate/up words.
    if (has_kv) fence_release_gpu();
    const Slice sl = slice_of(m, ly, nblk, 3, l, cta, ncta, geo.slot_bytes);
    if (sl.nrows == 0) return true;
    csync_();
    do_poll(Seg{fb.gt, stage, m.FF, G, m.FF, m.FF, act_mask(), tag(s, sid_gu(l))}, false);
    csync_();
    if (fail()) return false;
    tr_recv(s, sid_dn(l));
    const uint32_t tg = tag(s, sid_dn(l));
    gemv<false>(sl, stage, m.FF, m.FF, kEpiResid, l, tg);
    tr_done(s, sid_dn(l));
    return true;
  }

  // ------------------------------------------------------- head / sampler
  // Block statistics of this CTA's logits blocks (own logits in smem) for
  // the slots in `slots`: the logits to global memory (when `store`), and
  // per slot this CTA's greedy best and its max of s = l / T (the rules of
  // block_stats; both reductions are exact, so their grouping is free).
  __device__ void emit_stats(unsigned slots, uint32_t tg, bool store) {
    csync_();  // every warp's logits rows are in ol
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    ValIdx best[G];
    float smx[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
      best[g] = ValIdx{NAN, INT_MAX};
      smx[g] = -INFINITY;
    }
    for (int k = k0 + warp; k < k1; k += kPW) {
      const int i = k * kSBlk + lane;
      const bool valid = i < m.V;
#pragma unroll
      for (int g = 0; g < G; g++) {
        if (!((slots >> g) & 1u)) continue;
        const float l = valid ? ol[(size_t)g * geo.ol_f + (i - k0 * kSBlk)] : NAN;
        if (store && valid) bt.logits[(size_t)g * m.V + i] = l;
        const ValIdx bb = vi_warp_best(ValIdx{l, (valid && !isnan(l)) ? i : INT_MAX});
        if (vi_better(bb, best[g])) best[g] = bb;
        const float T = sh.sess[g].temperature;
        float sv = -INFINITY;
        if (valid && T != 0.0f) sv = __fdiv_rn(l, T);
        const float mr = warp_max(sv);
        smx[g] = fmaxf(smx[g], mr);
        if (T != 0.0f) {  // the row's statistics that steer the exact sampler's walk
          const float z = row_expsum(sv, valid, mr);
          if (lane == 0) {
            float* rm = reinterpret_cast<float*>(fb.esum) + (size_t)g * 2 * nblk;
            rm[k] = mr;
            rm[nblk + k] = z;
          }
        }
      }
    }
    if (lane == 0) {
#pragma unroll
      for (int g = 0; g < G; g++) {
        sh.wv[warp][g] = best[g].v;
        sh.wi[warp][g] = best[g].i;
        sh.ws[warp][g] = smx[g];
      }
    }
    csync_();
    if (threadIdx.x < G && ((slots >> threadIdx.x) & 1u)) {
      const int g = threadIdx.x;
      // the CTA's logits and row-statistics stores (before the barrier)
      // happen before these words: a sampling SELECT polls them with an
      // acquire, then reads both
      fence_release_gpu();
      ValIdx b{NAN, INT_MAX};
      float sm = -INFINITY;
      for (int w = 0; w < kPW; w++) {
        const ValIdx c{sh.wv[w][g], sh.wi[w][g]};
        if (vi_better(c, b)) b = c;
        sm = fmaxf(sm, sh.ws[w][g]);
      }
      uint64_t* cl = fb.cl + ((size_t)g * fb.cta_cap + cta) * 2;
      st_f(cl, b.v, tg);
      st_word(cl + 1, (uint32_t)b.i, tg);
      st_f(fb.csm + (size_t)g * fb.cta_cap + cta, sm, tg);
    }
    csync_();
  }

  __device__ bool head(int s) {
    tr_entry(s, sid_head(m.L));
    const Slice sl = slice_of(m, ly, nblk, 4, 0, cta, ncta, geo.slot_bytes);
    load_norm(m.norm);
    const unsigned act = act_mask();
    csync_();
    do_poll(Seg{fb.xt, stage, m.H, G, fb.xw, m.H, act, tag(s, sid_dn(m.L - 1))}, false);
    norm_ready();
    csync_();
    if (fail()) return false;
    tr_recv(s, sid_head(m.L));
    gemv<true>(sl, stage, m.H, m.H, kEpiHead, 0, 0u);
    emit_stats(act, tag(s, sid_head(m.L)), true);
    tr_done(s, sid_head(m.L));
    return true;
  }

  // The logits of the previous run (first step samples) as this CTA's own
  // logits, with their block statistics.
  __device__ void restat(unsigned slots) {
    const int n = (k1 - k0) * kSBlk;
#pragma unroll
    for (int g = 0; g < G; g++) {
      if (!((slots >> g) & 1u)) continue;
      for (int j = threadIdx.x; j < n; j += kPT) {
        const int i = k0 * kSBlk + j;
        ol[(size_t)g * geo.ol_f + j] = i < m.V ? ld_f(bt.logits + (size_t)g * m.V + i) : NAN;
      }
    }
    csync_();
    emit_stats(slots, tag(-1, sid_head(m.L)), false);
  }

  __device__ void finalize() {
    if (threadIdx.x != 0) return;
    for (int b = cta; b < bt.B; b += ncta) {
      DSlotState* st = sh.st + b;
      if (st->was_active) {
        st->pos += 1;
        st->step += 1;
      }
      st->was_active = 0;
      st->active = 0;
      if (st->step >= sh.sess[b].n_total) st->done = 1;
    }
  }

  __device__ void run(int nsteps) {
    unsigned first = 0;  // slots whose first step samples from the previous run's logits
    for (int g = 0; g < bt.B; g++) {
      const DSession& S = sh.sess[g];
      if (S.n_prompt == 0 && S.n_total > 0) first |= 1u << g;
    }
    if (first) restat(first);  // the greedy statistics of the previous run's logits
    for (int s = 0; s < nsteps; s++) {
      if (!select(s, first)) return;
      bool ended = false;
      for (int l = 0; l < m.L; l++) {
        if (!qkv(s, l)) {  // failure, or (at layer 0) no active slot
          ended = true;
          break;
        }
        if (!attn(s, l) || !oproj(s, l) || !gateup(s, l) || !down(s, l)) return;
      }
      if (ended) {
        if (fail()) return;
        break;
      }
      if (!head(s)) return;
      if (fail()) return;
    }
    finalize();
  }
};

template <bool BF16, int G>
__global__ void __launch_bounds__(kFlowThreads, 1)
    k_flow(const __grid_constant__ DModel m, const __grid_constant__ DBatch bt,
           const __grid_constant__ FlowBufs fb, const __grid_constant__ FlowGeo geo, int nsteps) {
  extern __shared__ __align__(1024) unsigned char fsm[];
  __shared__ FlowShared sh;
  const int tid = threadIdx.x, warp = tid >> 5;
  if (tid == 0) {
    for (int i = 0; i < geo.ring_slots; i++) {
      mbar_init(&sh.full[i], 1);
      mbar_init(&sh.empty[i], kPW);
    }
    sh.stop = 0;
    sh.fail = 0;
    sh.pfail = 0;
    sh.wait_ns = bt.wait_ns ? bt.wait_ns : kWaitNs;
    mbar_fence_init();
  }
  // Programs, slot state, stop lists and the layer table into shared memory.
  float* stage = reinterpret_cast<float*>(fsm + (size_t)geo.ring_slots * geo.slot_bytes);
  float* ol = stage + geo.stage_f;
  float* ownx = ol + (size_t)G * geo.ol_f;
  float* rope = ownx + (size_t)G * geo.ox_f;
  float* nw = rope + (size_t)G * geo.rope_f;
  DLayer* ly = reinterpret_cast<DLayer*>(nw + geo.res_f);
  if (tid < bt.B) {
    sh.sess[tid] = bt.sess[tid];
    sh.st[tid] = bt.st[tid];
    const int ns = min(sh.sess[tid].n_stop, kStopCache);
    for (int i = 0; i < ns; i++) sh.stops[tid][i] = sh.sess[tid].stop[i];
  }
  for (int i = tid; i < m.L; i += kFlowThreads) ly[i] = m.layers[i];
  __syncthreads();
  Ring rg{fsm, geo.ring_slots, geo.slot_bytes, sh.full, sh.empty, 0};
  const int cta = blockIdx.x, ncta = gridDim.x, nblk = bt.nblk;
  if (warp == kProducerWarp) {
    if ((tid & 31) == 0) produce(m, ly, nblk, rg, sh, nsteps, cta, ncta, bt.status);
    __syncwarp();
  } else {
    Flow<BF16, G> f{m, bt, fb, geo, sh, rg, cta, ncta, nblk, stages_per_step(m.L), stage, ol, ownx, rope, nw, ly,
                    0, 0, 0, 0, false};
    cta_range(nblk, cta, ncta, f.k0, f.k1);
    cta_range(m.H, cta, ncta, f.r0, f.r1);
    {
      int u0, u1;
      cta_range(m.QKVR / 2, cta, ncta, u0, u1);
      f.has_kv = u1 > u0 && 2 * u1 > m.QD;  // rows past the query rows are K/V rows
    }
    f.run(nsteps);
    DEFER_CTA_SYNC();
    // the owners' slot state back to global memory (also after a failure:
    // the host reads positions and divergences from it)
    if (tid < bt.B && tid % ncta == cta) bt.st[tid] = sh.st[tid];
    if (tid == 0) *(volatile int*)&sh.stop = 1;
  }
  __syncthreads();
}

}  // namespace

// ------------------------------------------------------------------- host
FlowPlan flow_plan(const DModel& m, int B, int max_chunks, int sms) {
  FlowPlan p;
  if (B < 1 || B > kMaxGroup) {
    p.why = "batch wider than the dataflow kernel's slot group";
    return p;
  }
  if (m.H % 8 || m.QD % 8 || m.FF % 8 || m.KVD % 8 || m.HD % 4 || m.HD != 2 * m.HALF || m.H > kNormRegs * kPT ||
      m.HALF > kPT) {
    p.why = "dimensions outside the dataflow kernel's layout";
    return p;
  }
  int dev = 0, optin = 0;
  DEFER_CUDA(cudaGetDevice(&dev));
  DEFER_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  const int G = group_of(B);
  const int ws = m.bf16 ? 2 : 4;
  const int nblk = (m.V + kSBlk - 1) / kSBlk;
  const int grid = std::min(sms, nblk);
  if (m.H < grid || m.FF < grid) {
    // every CTA must own gate/up and down rows: its tagged words of those
    // stages carry the release of its KV-cache appends to every other CTA
    p.why = "hidden or FFN width below the CTA count";
    return p;
  }
  const int Gh = m.NH / m.NKV;
  const size_t row_need = std::max({(size_t)2 * m.H * ws, (size_t)m.QD * ws, (size_t)m.FF * ws});
  const int SB = (int)std::max<size_t>(kSlotBytesMin, (row_need + 1023) & ~(size_t)1023);
  const int ol_f = kSBlk * ((nblk + grid - 1) / grid);
  const int ox_f = ((m.H + grid - 1) / grid + 3) & ~3;
  const int rope_f = 2 * m.HALF;
  const int nw_f = (m.H + 3) & ~3;  // norm weights of the current stage
  const int xw = header_words(m);
  const int ng2 = (nblk + 31) / 32, ng3 = (ng2 + 31) / 32;
  size_t st = (size_t)G * xw;
  st = std::max(st, (size_t)G * m.QD);
  st = std::max(st, (size_t)G * m.FF);
  st = std::max(st, (size_t)(Gh + 2) * m.HD + (size_t)Gh * kAttnChunk + (size_t)kAttnChunk * (m.HD + 4) +
                        (size_t)kAttnChunk * m.HD + Gh);
  st = std::max(st, (size_t)max_chunks * (m.HD + 2));
  st = std::max(st, (size_t)G * nblk + ng2 + ng3 + 8);
  st = std::max(st, (size_t)G * grid);
  st = std::max(st, (size_t)nblk + ng2 + ng3 + 8);
  st = std::max(st, (size_t)4 * grid);
  st = std::max(st, sample_exact_floats(m.V));  // the exact sampler of SELECT
  st = std::max(st, walk_records_floats(m.V));  // the owner's walk over every CTA's records
  st = (st + 31) & ~(size_t)31;
  const size_t rest = 4 * (st + (size_t)G * (ol_f + ox_f + rope_f) + nw_f) + (((size_t)m.L * sizeof(DLayer) + 15) & ~(size_t)15);
  const size_t budget = (size_t)optin > kStaticSmemReserve ? (size_t)optin - kStaticSmemReserve : 0;
  const int slots = budget > rest ? (int)std::min<size_t>(kMaxRing, (budget - rest) / SB) : 0;
  if (slots < 2) {
    p.why = "the weight ring does not fit in shared memory";
    return p;
  }
  p.geo.grid = grid;
  p.geo.ring_slots = slots;
  p.geo.slot_bytes = SB;
  p.geo.stage_f = (int)st;
  p.geo.ol_f = ol_f;
  p.geo.ox_f = ox_f;
  p.geo.rope_f = rope_f;
  p.geo.res_f = nw_f;
  p.geo.smem_bytes = (size_t)slots * SB + rest;
  p.ok = true;
  return p;
}

size_t flow_tagged_words(const DModel& m, int B, int max_chunks, int sms) {
  const int nblk = (m.V + kSBlk - 1) / kSBlk;
  const size_t xw = (size_t)header_words(m);
  return (size_t)B * (xw + (size_t)m.QD + 2 * m.KVD + m.QD + m.FF) +
         (size_t)B * m.NH * max_chunks * (m.HD + 2) + (size_t)B * sms * 3 + (size_t)B * nblk * 5 + (size_t)B;
}

FlowBufs flow_bufs(const DModel& m, int B, int max_chunks, int sms, uint64_t* w) {
  const int nblk = (m.V + kSBlk - 1) / kSBlk;
  FlowBufs f;
  f.xw = header_words(m);
  f.cta_cap = sms;
  f.xt = w;
  w += (size_t)B * f.xw;
  f.qt = w;
  w += (size_t)B * (m.QD + 2 * m.KVD);
  f.at = w;
  w += (size_t)B * m.QD;
  f.gt = w;
  w += (size_t)B * m.FF;
  f.pt = w;
  w += (size_t)B * m.NH * max_chunks * (m.HD + 2);
  f.cl = w;
  w += (size_t)B * sms * 2;
  f.csm = w;
  w += (size_t)B * sms;
  f.esum = w;
  w += (size_t)B * nblk;
  f.zrec = w;
  w += (size_t)B * nblk * 2;
  f.crec = w;
  w += (size_t)B * nblk * 2;
  f.invw = w;
  f.epoch = 1;
  return f;
}

int flow_stages_per_step(const DModel& m) { return stages_per_step(m.L); }

uint64_t flow_tags_per_run(const DModel& m, int nsteps) {
  return (uint64_t)(nsteps + 1) * (uint64_t)stages_per_step(m.L);
}

template <bool BF16, int G>
static void flow_impl(const DModel& m, const DBatch& bt, const FlowBufs& fb, const FlowGeo& geo, int nsteps,
                      cudaStream_t st) {
  auto kern = k_flow<BF16, G>;
  DEFER_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)geo.smem_bytes));
  int per_sm = 0;
  DEFER_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kFlowThreads, geo.smem_bytes));
  if (per_sm < 1) fail(kCuda, "dataflow token-loop kernel cannot be resident");
  DModel mm = m;
  DBatch bb = bt;
  FlowBufs ff = fb;
  FlowGeo gg = geo;
  int ns = nsteps;
  void* args[] = {&mm, &bb, &ff, &gg, &ns};
  DEFER_CUDA(cudaLaunchCooperativeKernel((const void*)kern, dim3(geo.grid), dim3(kFlowThreads), args,
                                         geo.smem_bytes, st));
}

void launch_steps_flow(const DModel& m, const DBatch& bt, const FlowBufs& fb, const FlowPlan& plan, int nsteps,
                       cudaStream_t st) {
  if (!plan.ok) fail(kInvalidArgument, std::string("dataflow kernel not applicable: ") + plan.why);
  const int G = group_of(bt.B);
  if (m.bf16) {
    switch (G) {
      case 1: flow_impl<true, 1>(m, bt, fb, plan.geo, nsteps, st); break;
      case 2: flow_impl<true, 2>(m, bt, fb, plan.geo, nsteps, st); break;
      case 4: flow_impl<true, 4>(m, bt, fb, plan.geo, nsteps, st); break;
      default: flow_impl<true, 8>(m, bt, fb, plan.geo, nsteps, st); break;
    }
  } else {
    switch (G) {
      case 1: flow_impl<false, 1>(m, bt, fb, plan.geo, nsteps, st); break;
      case 2: flow_impl<false, 2>(m, bt, fb, plan.geo, nsteps, st); break;
      case 4: flow_impl<false, 4>(m, bt, fb, plan.geo, nsteps, st); break;
      default: flow_impl<false, 8>(m, bt, fb, plan.geo, nsteps, st); break;
    }
  }
}

}  // namespace defer

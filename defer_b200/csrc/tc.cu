// Tensor-core (tcgen05) contraction of wide batched steps that never sample
// (the leave-one-out attribution batch, attribution.rs:224-264): every
// projection of the step is one GEMM Y[slot][row] = A[slot][k] . W[row][k]
// over up to 128 slots, on the 5th-generation tensor cores with the
// accumulator in tensor memory.
//
// Precision. The activations are fp32 and split into bf16 terms, x_hi =
// bf16(x), x_mid = bf16(x - x_hi), x_lo = bf16(x - x_hi - x_mid) (each
// residual exact in fp32). Weights stored as bf16 are exact in one term:
// the product is x_hi.w + x_mid.w + x_lo.w, off by at most 2^-27 of each
// term's magnitude (below fp32's own rounding). fp32 weights are split in
// two, w_hi + w_lo, and the activations in two: x_hi.w_hi + x_hi.w_lo +
// x_lo.w_hi with x_lo = bf16(x - x_hi), within 2^-17 of each product.
// Accumulation is fp32 in tensor memory. Results are checked against the CPU oracle at
// the parity tolerance; they are deterministic run to run (fixed K-block
// order, split-K partial sums added in split order), but not bit-identical
// to the CUDA-core path of the other token loops.
//
// Operand layout. Both operands are K-major bf16 in the canonical layout
// without swizzle: 8 x 8 core matrices (8 rows of 16 bytes, 128 contiguous
// bytes), a 64-wide K block of R rows stored as (row group g, k chunk c) at
// (g * 8 + c) * 128 bytes, so the leading byte offset (next k chunk) is 128
// and the stride byte offset (next row group) is 1024. Activations of one
// K block: [hi][mid][lo] or [hi][lo], 128 rows each (16 KB per term);
// weights are packed once into tiles of 128 rows x 64 k, [hi][lo] per tile
// (32 KB, 16 KB when bf16), ordered row tile major, K block minor, so a
// CTA's K range is contiguous.
//
// GEMM kernel (k_tc_gemm): one CTA per (128-row tile, K split); 6 warps.
// Warp 4 streams A and W blocks with bulk copies into a 3-stage ring of
// 64 KB stages (mbarrier complete_tx); warp 5 issues the MMAs (M = 128,
// N = 128, K = 16 per instruction, 3 products per k step) and commits each
// stage back to the producer. The tensor core's own fp32 accumulation loses accuracy over
// long chains (on the 8B widths a 32-block chain was ~10x less accurate than
// fp32 dot products), so the K range is cut into groups of kTcGroup blocks:
// each group accumulates from zero into one of two TMEM buffers, and warps
// 0-3 read it (tcgen05.ld, TMEM lane = slot) and add it into registers in
// group order while the next group runs in the other buffer; they store the
// 128 partial sums at the end. A 128-row tile reads the activation block
// once per 128 weight rows: with fp32 weights the bytes a CTA brings in
// are half weights, half activations (a 64-row tile: one third weights).
// Every wait is bounded; a wait that runs out sets the status word, the CTA
// drains its copies and MMAs in flight and frees its tensor memory.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <vector>

#include "common.h"
#include "kernels.h"
#include "phases.cuh"
#include "tc.h"

namespace defer {
namespace {

constexpr int kTcBN = 128;                       // weight rows per tile (MMA N)
constexpr int kTcBK = 64;                        // K per block
constexpr int kTcStages = 3;
constexpr int kTcABytes = kTcM * kTcBK * 2;      // one bf16 term of an activation block
constexpr int kTcWBytes = kTcBN * kTcBK * 2;     // one bf16 term of a weight tile
constexpr int kTcStageMax = 3 * kTcABytes + kTcWBytes;  // the largest stage: 3 + 1 terms (2 + 2 is the same)
constexpr int kTcThreads = 192;  // warps 0-3 drain TMEM, 4 copies, 5 issues MMAs
constexpr int kTcGroup = 4;      // K blocks per tensor-core accumulation chain
constexpr unsigned long long kTcWaitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mb_init(uint64_t* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mb_expect_tx(uint64_t* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mb_try(uint64_t* b, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(saddr(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase of `parity` to complete; false when it ran out.
__device__ __forceinline__ bool mb_wait(uint64_t* b, unsigned parity) {
  if (mb_try(b, parity)) return true;
  const unsigned long long t0 = gtime();
  unsigned spins = 0;
  while (!mb_try(b, parity)) {
    if ((++spins & 63u) == 0 && gtime() - t0 > kTcWaitNs) return false;
  }
  return true;
}
__device__ __forceinline__ void bulk_copy(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   saddr(dst)),
               "l"(src), "r"(bytes), "r"(saddr(bar))
               : "memory");
}

// Shared-memory matrix descriptor: K-major, no swizzle, Blackwell version.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version 1; base offset 0, layout SWIZZLE_NONE
  return d;
}
// Instruction descriptor of kind::f16: bf16 A and B (both K-major), fp32 D.
constexpr uint32_t kIdesc = (1u << 4)                       // D format f32
                            | (1u << 7) | (1u << 10)        // A, B format bf16
                            | ((uint32_t)(kTcBN >> 3) << 17)  // N
                            | ((uint32_t)(kTcM >> 4) << 24);  // M

__device__ __forceinline__ void umma(uint32_t dtm, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(dtm), "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(bar))
               : "memory");
}

struct TcGemmArgs {
  const unsigned char* A;  // [nkb][aterms][kTcM * kTcBK] bf16
  const unsigned char* W;  // [ntile][nkb][wterms][kTcBN * kTcBK] bf16
  float* Y;                // [splits][kTcM][n_pad] partial sums; the total in split 0's rows
  unsigned* tickets;       // [ntile] splits of the tile finished
  int nkb, splits, n_pad, wterms, aterms;  // aterms = 3 when wterms = 1, else 2
  int* status;
  const int* active;  // the step's "any slot active" flag, or null (always run)
};

__device__ __forceinline__ void mb_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(b)) : "memory");
}

__global__ void __launch_bounds__(kTcThreads, 1) k_tc_gemm(const __grid_constant__ TcGemmArgs g) {
  extern __shared__ __align__(1024) unsigned char tsm[];
  __shared__ __align__(8) uint64_t full[kTcStages], empty[kTcStages], acc_full[2], acc_empty[2], drain;
  __shared__ uint32_t tmem_base;
  __shared__ int failed, last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (g.active && __ldcg(g.active) == 0) return;  // no slot fed a token this step
  const int tile = blockIdx.x / g.splits, sp = blockIdx.x % g.splits;
  const int kb0 = sp * g.nkb / g.splits, kb1 = (sp + 1) * g.nkb / g.splits;
  const int nk = kb1 - kb0;
  const int ngroups = (nk + kTcGroup - 1) / kTcGroup;
  unsigned char* ring = tsm;
  if (tid == 0) {
    for (int s = 0; s < kTcStages; s++) {
      mb_init(&full[s], 1);
      mb_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mb_init(&acc_full[b], 1);
      mb_init(&acc_empty[b], 4);  // one arrival per draining warp
    }
    mb_init(&drain, 1);
    failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 5) {  // two 128 x 128 fp32 accumulators: 256 columns of tensor memory
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(&tmem_base)),
                 "r"(2 * kTcBN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tm = tmem_base;
  const size_t wtile = (size_t)g.wterms * kTcWBytes;
  const unsigned a_bytes = (unsigned)g.aterms * kTcABytes;
  const unsigned stage_bytes = a_bytes + (unsigned)wtile;  // a multiple of 1024

  float acc[kTcBN];  // the draining warps' sums (slot = TMEM lane, one row tile)
#pragma unroll
  for (int c = 0; c < kTcBN; c++) acc[c] = 0.0f;
  if (warp == 4) {
    if (lane == 0) {
      // producer: this CTA's K blocks of A and of its weight tile
      int issued = 0;
      for (int i = 0; i < nk; i++) {
        const int s = i % kTcStages;
        if (i >= kTcStages && !mb_wait(&empty[s], (unsigned)((i / kTcStages - 1) & 1))) {
          atomicCAS(g.status, kStOk, kStTimeout);
          *(volatile int*)&failed = 1;
          break;
        }
        if (*(volatile int*)&failed) break;
        unsigned char* st = ring + (size_t)s * stage_bytes;
        mb_expect_tx(&full[s], stage_bytes);
        bulk_copy(st, g.A + (size_t)(kb0 + i) * a_bytes, a_bytes, &full[s]);
        bulk_copy(st + a_bytes, g.W + ((size_t)tile * g.nkb + kb0 + i) * wtile, (unsigned)wtile, &full[s]);
        issued = i + 1;
      }
      // copies still in flight land before the CTA leaves: the last one of each stage
      for (int i = max(0, issued - kTcStages); i < issued; i++)
        if (!mb_wait(&full[i % kTcStages], (unsigned)((i / kTcStages) & 1))) atomicCAS(g.status, kStOk, kStTimeout);
    }
  } else if (warp == 5) {
    if (lane == 0) {
      // MMA issuer: group gi of kTcGroup K blocks accumulates from zero into
      // buffer gi & 1, which the draining warps empty while the next group runs
      bool ok = true;
      int i = 0;
      for (int gi = 0; gi < ngroups && ok; gi++) {
        const int buf = gi & 1;
        if (gi >= 2 && !mb_wait(&acc_empty[buf], (unsigned)(((gi >> 1) - 1) & 1))) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tm + (uint32_t)(buf * kTcBN);
        const int i0 = gi * kTcGroup, iend = min(nk, i0 + kTcGroup);
        for (i = i0; i < iend; i++) {
          const int s = i % kTcStages;
          if (!mb_wait(&full[s], (unsigned)((i / kTcStages) & 1))) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t st = saddr(ring + (size_t)s * stage_bytes);
          const uint32_t a_hi = st, a_2 = st + kTcABytes, w_hi = st + a_bytes, w_lo = w_hi + kTcWBytes;
#pragma unroll
          for (int ks = 0; ks < kTcBK / 16; ks++) {
            const uint32_t o = (uint32_t)ks * 256u;  // two 8-wide k chunks of 128 bytes each
            const uint64_t ah = smem_desc(a_hi + o, 128, 1024), a2 = smem_desc(a_2 + o, 128, 1024);
            const uint64_t wh = smem_desc(w_hi + o, 128, 1024);
            umma(d, ah, wh, (i > i0 || ks > 0) ? 1u : 0u);
            umma(d, a2, wh, 1u);  // x_mid (3 terms) or x_lo (2 terms) times w_hi
            if (g.wterms == 2) umma(d, ah, smem_desc(w_lo + o, 128, 1024), 1u);
            else umma(d, smem_desc(a_2 + kTcABytes + o, 128, 1024), wh, 1u);  // x_lo times w
          }
          umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
      if (!ok) {
        atomicCAS(g.status, kStOk, kStTimeout);
        *(volatile int*)&failed = 1;
      }
      // every MMA issued has completed before tensor memory is freed
      umma_commit(&drain);
      if (!mb_wait(&drain, 0u)) atomicCAS(g.status, kStOk, kStTimeout);
    }
  } else {
    // warps 0-3: lane r of TMEM = slot r; each group's 128 partial sums are
    // added into registers in group order (fp32, round to nearest), which
    // keeps every tensor-core accumulation chain to kTcGroup K blocks
    bool ok = true;
    for (int gi = 0; gi < ngroups; gi++) {
      const int buf = gi & 1;
      // the warp-collective TMEM loads need one decision per warp
      ok = __all_sync(0xffffffffu, mb_wait(&acc_full[buf], (unsigned)((gi >> 1) & 1)));
      if (!ok) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
      for (int c0 = 0; c0 < kTcBN; c0 += 16) {
        uint32_t v[16];
        const uint32_t ta = tm + ((uint32_t)(warp * 32) << 16) + (uint32_t)(buf * kTcBN + c0);
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
            : "r"(ta));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int j = 0; j < 16; j++) acc[c0 + j] = __fadd_rn(acc[c0 + j], __uint_as_float(v[j]));
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mb_arrive(&acc_empty[buf]);
    }
    if (!ok) {
      if (lane == 0) atomicCAS(g.status, kStOk, kStTimeout);
      *(volatile int*)&failed = 1;
    } else if (g.splits > 1) {
      const int r = warp * 32 + lane;  // an empty K range stores zeros
      float* y = g.Y + ((size_t)sp * kTcM + r) * g.n_pad + (size_t)tile * kTcBN;
#pragma unroll
      for (int c = 0; c < kTcBN; c += 4)
        *reinterpret_cast<float4*>(y + c) = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
      __threadfence();  // this split's partials before its ticket
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (g.splits > 1 && tid == 0) {
    const unsigned t = atomicAdd(g.tickets + tile, 1u);
    last = t == (unsigned)g.splits - 1;
    if (last) g.tickets[tile] = 0;  // every split has counted: zero for the next GEMM
  }
  __syncthreads();
  if (warp < 4 && !*(volatile int*)&failed && (g.splits == 1 || last)) {
    // the tile's total, the splits added in split order (this split's own
    // partials from registers), into split 0's rows
    if (g.splits > 1) __threadfence();
    const int r = warp * 32 + lane;
    float* y0 = g.Y + (size_t)r * g.n_pad + (size_t)tile * kTcBN;
#pragma unroll
    for (int c = 0; c < kTcBN; c += 4) {
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int q = 0; q < g.splits; q++) {
        float4 p;
        if (q == sp) p = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
        else p = __ldcg(reinterpret_cast<const float4*>(g.Y + ((size_t)q * kTcM + r) * g.n_pad + (size_t)tile * kTcBN + c));
        if (q == 0) {
          t = p;
        } else {
          t.x = __fadd_rn(t.x, p.x);
          t.y = __fadd_rn(t.y, p.y);
          t.z = __fadd_rn(t.z, p.z);
          t.w = __fadd_rn(t.w, p.w);
        }
      }
      *reinterpret_cast<float4*>(y0 + c) = t;
    }
  }
  __syncthreads();
  if (warp == 5) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(2 * kTcBN) : "memory");
  }
}

// Offset (elements) of (row r, k) inside one 64-wide K block of R rows.
__host__ __device__ __forceinline__ size_t core_off(int r, int kk) {
  return ((size_t)((r >> 3) * 8 + (kk >> 3)) << 6) + (size_t)((r & 7) << 3) + (size_t)(kk & 7);
}

__device__ __forceinline__ void split_bf16(float x, __nv_bfloat16& hi, __nv_bfloat16& lo) {
  hi = __float2bfloat16_rn(x);
  lo = __float2bfloat16_rn(__fsub_rn(x, __bfloat162float(hi)));
}
__device__ __forceinline__ void split3_bf16(float x, __nv_bfloat16& hi, __nv_bfloat16& mid, __nv_bfloat16& lo) {
  hi = __float2bfloat16_rn(x);
  const float r = __fsub_rn(x, __bfloat162float(hi));
  mid = __float2bfloat16_rn(r);
  lo = __float2bfloat16_rn(__fsub_rn(r, __bfloat162float(mid)));
}

// Weight packing: W [N][K] (fp32, or bf16 when `bf16`) -> tiles; one thread
// per 8-wide k chunk of one row. Rows >= N and k >= K are zero.
__global__ void k_tc_pack_w(const void* W, int N, int K, int bf16, int nkb, int wterms, unsigned char* out,
                            size_t chunks) {
  for (size_t c = blockIdx.x * (size_t)blockDim.x + threadIdx.x; c < chunks; c += (size_t)gridDim.x * blockDim.x) {
    const int kc = (int)(c % (size_t)(nkb * 8));
    const int n = (int)(c / (size_t)(nkb * 8));
    const int k0 = kc * 8;
    __align__(16) __nv_bfloat16 hi[8], lo[8];
#pragma unroll
    for (int e = 0; e < 8; e++) {
      const int k = k0 + e;
      float x = 0.0f;
      if (n < N && k < K) {
        if (bf16)
          x = __uint_as_float((uint32_t)(reinterpret_cast<const uint16_t*>(W)[(size_t)n * K + k]) << 16);
        else
          x = reinterpret_cast<const float*>(W)[(size_t)n * K + k];
      }
      split_bf16(x, hi[e], lo[e]);
    }
    const int tile = n / kTcBN, r = n % kTcBN, kb = k0 / kTcBK, kk = k0 % kTcBK;
    unsigned char* t = out + ((size_t)tile * nkb + kb) * (size_t)wterms * kTcWBytes;
    *reinterpret_cast<uint4*>(t + core_off(r, kk) * 2) = *reinterpret_cast<const uint4*>(hi);
    if (wterms == 2) *reinterpret_cast<uint4*>(t + kTcWBytes + core_off(r, kk) * 2) = *reinterpret_cast<const uint4*>(lo);
  }
}

// The 8 values at k0.. of one A row, split into `aterms` bf16 terms and
// stored in the operand's core-matrix layout.
__device__ __forceinline__ void put_a_chunk(unsigned char* A, int b, int k0, const float* v, int aterms) {
  __align__(16) __nv_bfloat16 hi[8], mid[8], lo[8];
#pragma unroll
  for (int e = 0; e < 8; e++) {
    if (aterms == 3) split3_bf16(v[e], hi[e], mid[e], lo[e]);
    else split_bf16(v[e], hi[e], mid[e]);  // [hi][lo]: the second term in mid
  }
  const int kb = k0 / kTcBK, kk = k0 % kTcBK;
  unsigned char* blk = A + (size_t)kb * aterms * kTcABytes;
  *reinterpret_cast<uint4*>(blk + core_off(b, kk) * 2) = *reinterpret_cast<const uint4*>(hi);
  *reinterpret_cast<uint4*>(blk + kTcABytes + core_off(b, kk) * 2) = *reinterpret_cast<const uint4*>(mid);
  if (aterms == 3)
    *reinterpret_cast<uint4*>(blk + 2 * kTcABytes + core_off(b, kk) * 2) = *reinterpret_cast<const uint4*>(lo);
}

// Slot row b of the A operand from row xr ([K]), RMS-normalised with weight
// `nw` when nw != null ((x * inv) * w, inv = 1 / sqrt(ss / K + eps) with ss
// a fixed-tree sum: thread t's fmaf chain over k = t, t + 256, ..., warp
// butterfly, warps in order), split into `aterms` bf16 terms; zero when the
// slot is not live. A whole 256-thread CTA; a thread's first loop reads only
// the k = t + 256 j it may itself have just written.
__device__ __forceinline__ void prep_row(const float* xr, const float* nw, float eps, int K, int nkb, bool live, int b,
                                         unsigned char* A, int aterms) {
  const int tid = threadIdx.x;
  __shared__ float red[8];
  __shared__ float s_inv;
  if (nw && live) {
    float acc = 0.0f;
    for (int k = tid; k < K; k += 256) {
      const float v = __ldcg(xr + k);
      acc = fmaf(v, v, acc);
    }
    acc = warp_sum_butterfly(acc);
    if ((tid & 31) == 0) red[tid >> 5] = acc;
    __syncthreads();
    if (tid == 0) {
      float ss = 0.0f;
      for (int w = 0; w < 8; w++) ss = __fadd_rn(ss, red[w]);
      s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));
    }
    __syncthreads();
  }
  const float inv = (nw && live) ? s_inv : 1.0f;
  const int kpad = nkb * kTcBK;
  for (int k0 = tid * 8; k0 < kpad; k0 += 256 * 8) {
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; e++) {
      const int k = k0 + e;
      v[e] = 0.0f;
      if (live && k < K) {
        v[e] = __ldcg(xr + k);
        if (nw) v[e] = __fmul_rn(__fmul_rn(v[e], inv), nw[k]);
      }
    }
    put_a_chunk(A, b, k0, v, aterms);
  }
}

// Activations -> A blocks: slot row b (one CTA each, 128 of them) of `x`
// ([B][K], row stride K). Rows of slots >= B or not active are zero.
__global__ void __launch_bounds__(256) k_tc_prep(const float* x, const float* nw, float eps, int K, int nkb, int B,
                                                 const DSlotState* st, unsigned char* A, const int* active,
                                                 int aterms) {
  const int b = blockIdx.x;
  if (active && __ldcg(active) == 0) return;
  const bool live = b < B && __ldcg(&st[b].active) != 0;
  prep_row(x + (size_t)b * K, nw, eps, K, nkb, live, b, A, aterms);
}

// Sum of the split-K partials of (slot b, column n), in split order.
__device__ __forceinline__ float ysum(const float* Y, int splits, int n_pad, int b, int n) {
  float v = Y[(size_t)b * n_pad + n];
  for (int s = 1; s < splits; s++) v = __fadd_rn(v, Y[((size_t)s * kTcM + b) * n_pad + n]);
  return v;
}

__device__ __forceinline__ bool live_slot(const DBatch& bt, int b) { return ld_i(&bt.st[b].active) != 0; }

// QKV epilogue: pair u (rows 2u, 2u+1) of slot b -> bias, RoPE, q / KV append.
__global__ void k_tc_qkv_epi(DModel m, DBatch bt, int l, const float* Y, int splits, int n_pad) {
  const DLayer& Ly = m.layers[l];
  const int pairs = m.QKVR / 2;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < bt.B * pairs; i += gridDim.x * blockDim.x) {
    const int b = i / pairs, u = i - b * pairs;
    if (!live_slot(bt, b)) continue;
    const float a = ysum(Y, splits, n_pad, b, 2 * u), c = ysum(Y, splits, n_pad, b, 2 * u + 1);
    qkv_store(m, Ly, bt, l, u, b, ld_i(&bt.st[b].pos), a, c);
  }
}

// x[b] += Y (the O or down projection's total), then slot row b of the next
// projection's A operand from the updated row, normalised with `nw` (the
// next RMSNorm's weights): one launch and one pass over x instead of a
// residual kernel and a prep. One CTA per slot.
__global__ void __launch_bounds__(256) k_tc_resid_prep(DModel m, DBatch bt, const float* __restrict__ Y, int n_pad,
                                                       const float* nw, int nkb, unsigned char* A,
                                                       const int* active, int aterms) {
  const int b = blockIdx.x, tid = threadIdx.x;
  if (active && __ldcg(active) == 0) return;
  const bool live = b < bt.B && live_slot(bt, b);
  float* __restrict__ xr = bt.x + (size_t)b * m.H;
  const float* __restrict__ yr = Y + (size_t)b * n_pad;
  if (live) {
#pragma unroll 4
    for (int k = tid; k < m.H; k += 256) xr[k] = __fadd_rn(__ldcg(xr + k), __ldcg(yr + k));
  }
  __syncthreads();
  prep_row(xr, nw, m.eps, m.H, nkb, live, b, A, aterms);
}

// g = act(gate) * up of slot row b (gate and up interleaved in Y), straight
// into the down projection's A operand (g itself is not stored). Grid:
// (slot, 2048-wide slice of g).
__global__ void __launch_bounds__(256) k_tc_gu_prep(DModel m, DBatch bt, const float* __restrict__ Y, int n_pad,
                                                    int nkb, unsigned char* A, const int* active, int aterms) {
  const int b = blockIdx.x;
  if (active && __ldcg(active) == 0) return;
  const bool live = b < bt.B && live_slot(bt, b);
  const int k0 = (blockIdx.y * 256 + threadIdx.x) * 8;
  if (k0 >= nkb * kTcBK) return;
  float v[8];
  if (live && k0 + 8 <= m.FF) {
    const float4* yp = reinterpret_cast<const float4*>(Y + (size_t)b * n_pad + 2 * (size_t)k0);
    float4 q[4];
#pragma unroll
    for (int e = 0; e < 4; e++) q[e] = __ldcg(yp + e);
#pragma unroll
    for (int e = 0; e < 4; e++) {
      v[2 * e] = gate_act_mul(m, q[e].x, q[e].y);
      v[2 * e + 1] = gate_act_mul(m, q[e].z, q[e].w);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; e++) {
      const int j = k0 + e;
      v[e] = (live && j < m.FF) ? gate_act_mul(m, __ldcg(Y + (size_t)b * n_pad + 2 * j),
                                               __ldcg(Y + (size_t)b * n_pad + 2 * j + 1))
                                : 0.0f;
    }
  }
  put_a_chunk(A, b, k0, v, aterms);
}

__global__ void k_tc_head_epi(DModel m, DBatch bt, const float* Y, int splits, int n_pad) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (size_t)bt.B * m.V;
       i += (size_t)gridDim.x * blockDim.x) {
    const int b = (int)(i / m.V), n = (int)(i - (size_t)b * m.V);
    if (!live_slot(bt, b)) continue;
    bt.logits[(size_t)b * m.V + n] = ysum(Y, splits, n_pad, b, n);
  }
}

// Greedy block statistics of the new logits (a greedy SELECT reads them).
__global__ void __launch_bounds__(kThreads) k_tc_stats(DModel m, DBatch bt) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = bt.nblk;
  for (size_t u = (size_t)blockIdx.x * kPW + warp; u < (size_t)bt.B * nb; u += (size_t)gridDim.x * kPW) {
    const int b = (int)(u / nb), k = (int)(u - (size_t)b * nb);
    if (!live_slot(bt, b)) continue;
    const int i = k * kSBlk + lane;
    const bool valid = i < m.V;
    const size_t o = (size_t)b * nb + k;
    block_stats(valid ? ld_f(bt.logits + (size_t)b * m.V + i) : NAN, i, valid, bt.sess[b].temperature,
                bt.ss.lmax + o, bt.ss.larg + o, bt.ss.smax + o, bt.ss.esum + o);
  }
}
__global__ void __launch_bounds__(kThreads) k_tc_restat(DModel m, DBatch bt) {
  ph_restat(m, bt, blockIdx.x, gridDim.x);
}

// The step's phases that stay on the CUDA cores.
template <bool BF16>
__global__ void __launch_bounds__(kThreads) k_tc_select(DModel m, DBatch bt, int run_step) {
  extern __shared__ __align__(16) float tsel[];
  ph_select<BF16>(m, bt, run_step, blockIdx.x, gridDim.x, tsel);
}
__global__ void __launch_bounds__(kThreads) k_tc_attn(DModel m, DBatch bt, int l) {
  extern __shared__ __align__(16) float tat[];
  ph_attn_chunks(m, bt, l, blockIdx.x, gridDim.x, tat);
}
__global__ void __launch_bounds__(kThreads) k_tc_combine(DModel m, DBatch bt) {
  ph_attn_combine(m, bt, blockIdx.x, gridDim.x);
}
__global__ void __launch_bounds__(kThreads) k_tc_finalize(DBatch bt) { ph_finalize(bt, blockIdx.x, gridDim.x); }

int div_up(long a, long b) { return (int)((a + b - 1) / b); }

}  // namespace

// ----------------------------------------------------------------- host
size_t tc_packed_bytes(int N, int K, bool bf16) {
  const size_t nt = (size_t)div_up(N, kTcBN), nkb = (size_t)div_up(K, kTcBK);
  return nt * nkb * (bf16 ? 1 : 2) * (size_t)kTcWBytes;
}

TcMatrix tc_pack(const void* W, int N, int K, bool bf16, unsigned char* out, cudaStream_t st) {
  TcMatrix t;
  t.N = N;
  t.K = K;
  t.nkb = div_up(K, kTcBK);
  t.ntile = div_up(N, kTcBN);
  t.wterms = bf16 ? 1 : 2;
  t.data = out;
  const size_t chunks = (size_t)t.ntile * kTcBN * t.nkb * 8;
  k_tc_pack_w<<<std::min<size_t>((chunks + 255) / 256, 148 * 16), 256, 0, st>>>(W, N, K, bf16 ? 1 : 0, t.nkb,
                                                                               t.wterms, out, chunks);
  DEFER_CUDA(cudaGetLastError());
  return t;
}

size_t tc_act_bytes(int K) { return (size_t)div_up(K, kTcBK) * 3 * kTcABytes; }

int tc_aterms(const TcMatrix& w) { return w.wterms == 1 ? 3 : 2; }

void tc_prep(const float* x, const float* nw, float eps, int K, int B, const DSlotState* st, unsigned char* A,
             int aterms, cudaStream_t s, const int* active) {
  if (aterms != 2 && aterms != 3) fail(kInvalidArgument, "tensor-core step: activation terms must be 2 or 3");
  k_tc_prep<<<kTcM, 256, 0, s>>>(x, nw, eps, K, div_up(K, kTcBK), B, st, A, active, aterms);
  DEFER_CUDA(cudaGetLastError());
}

int tc_splits(const TcMatrix& w, int sms) {
  // The last split of a tile reads the other splits' 64 KB partials, so s
  // splits cost a tile about W/s + (s - 1) * 64 KB of one SM's reads (W the
  // tile's weight bytes): s near sqrt(W / 64 KB); at most one wave of CTAs
  // (one CTA per SM) and at least 4 K blocks a split.
  const double wtile = (double)kTcBN * w.K * 2.0 * w.wterms;
  const int best = (int)std::lround(std::sqrt(wtile / (64.0 * 1024.0)));
  return std::max(1, std::min({sms / std::max(1, w.ntile), w.nkb / 4, best}));
}

// Kernel attributes are set once per device.
static bool first_on_device(unsigned long long& mask) {
  int dev = 0;
  DEFER_CUDA(cudaGetDevice(&dev));
  const unsigned long long bit = 1ull << (dev & 63);
  if (mask & bit) return false;
  mask |= bit;
  return true;
}

void tc_gemm(const unsigned char* A, const TcMatrix& w, float* Y, int splits, unsigned* tickets, int* status,
             cudaStream_t s, const int* active) {
  static unsigned long long attr = 0;
  if (first_on_device(attr))
    DEFER_CUDA(cudaFuncSetAttribute(k_tc_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    kTcStages * kTcStageMax));
  const int smem = kTcStages * (tc_aterms(w) * kTcABytes + w.wterms * kTcWBytes);
  TcGemmArgs g;
  g.A = A;
  g.W = w.data;
  g.Y = Y;
  g.tickets = tickets;
  g.nkb = w.nkb;
  g.splits = splits;
  g.n_pad = w.ntile * kTcBN;
  g.wterms = w.wterms;
  g.aterms = tc_aterms(w);
  g.status = status;
  g.active = active;
  k_tc_gemm<<<w.ntile * splits, kTcThreads, smem, s>>>(g);
  DEFER_CUDA(cudaGetLastError());
}

size_t tc_y_floats(const TcMatrix& w, int splits) { return (size_t)splits * kTcM * w.ntile * kTcBN; }

void launch_steps_tc(const DModel& m, const TcModel& tm, const DBatch& bt0, int nsteps, int sms, TcWork& wk,
                     cudaStream_t st) {
  if (bt0.B > kTcM) fail(kInvalidArgument, "tensor-core step: more than 128 slots");
  DBatch bt = bt0;
  const size_t smem = step_smem_bytes(m, bt.B, bt.max_chunks);
  bt.smem_bytes = (unsigned)smem;
  bt.parts = 1;
  static unsigned long long attr = 0;
  if (first_on_device(attr)) {
    DEFER_CUDA(cudaFuncSetAttribute(k_tc_select<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    DEFER_CUDA(cudaFuncSetAttribute(k_tc_select<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    DEFER_CUDA(cudaFuncSetAttribute(k_tc_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
  }
  if (smem > 200 * 1024) fail(kInvalidArgument, "tensor-core step: phase shared memory too large");
  const int attn_units = bt.B * m.NKV * bt.max_chunks;
  const int ew = std::min(sms * 8, 4096);  // epilogue grid
  const int nb = bt.nblk;
  // statistics of the resident logits for slots whose first step samples
  k_tc_restat<<<std::min(sms, std::max(1, nb / kPW)), kThreads, 0, st>>>(m, bt);
  const int at = tc_aterms(tm.head);  // the model's weights share one type
  const int nkb_h = div_up(m.H, kTcBK), nkb_ff = div_up(m.FF, kTcBK);
  for (int s = 0; s < nsteps; s++) {
    if (m.bf16) k_tc_select<true><<<bt.B, kThreads, smem, st>>>(m, bt, s);
    else k_tc_select<false><<<bt.B, kThreads, smem, st>>>(m, bt, s);
    const int* act = bt.any_active + (s & 1);  // set by this step's SELECT
    tc_prep(bt.x, tm.layers[0].attn_norm, m.eps, m.H, bt.B, bt.st, wk.A, at, st, act);
    for (int l = 0; l < m.L; l++) {
      const TcLayer& T = tm.layers[l];
      // the A operand of QKV is ready (the step's first prep, or the last
      // layer's residual)
      tc_gemm(wk.A, T.qkv, wk.Y, T.s_qkv, wk.tickets, bt.status, st, act);
      k_tc_qkv_epi<<<ew, 256, 0, st>>>(m, bt, l, wk.Y, 1, T.qkv.ntile * kTcBN);
      k_tc_attn<<<std::min(attn_units, sms * 8), kThreads, smem, st>>>(m, bt, l);
      k_tc_combine<<<sms, kThreads, 0, st>>>(m, bt);
      tc_prep(bt.att, nullptr, 0.0f, m.QD, bt.B, bt.st, wk.A, at, st, act);
      tc_gemm(wk.A, T.o, wk.Y, T.s_o, wk.tickets, bt.status, st, act);
      k_tc_resid_prep<<<kTcM, 256, 0, st>>>(m, bt, wk.Y, T.o.ntile * kTcBN, T.ffn_norm, nkb_h, wk.A, act, at);
      tc_gemm(wk.A, T.gu, wk.Y, T.s_gu, wk.tickets, bt.status, st, act);
      k_tc_gu_prep<<<dim3(kTcM, div_up((long)nkb_ff * kTcBK, 2048)), 256, 0, st>>>(m, bt, wk.Y, T.gu.ntile * kTcBN,
                                                                            nkb_ff, wk.A, act, at);
      tc_gemm(wk.A, T.down, wk.Y, T.s_down, wk.tickets, bt.status, st, act);
      const float* next_norm = l + 1 < m.L ? tm.layers[l + 1].attn_norm : m.norm;
      k_tc_resid_prep<<<kTcM, 256, 0, st>>>(m, bt, wk.Y, T.down.ntile * kTcBN, next_norm, nkb_h, wk.A, act,
                                           at);
    }
    tc_gemm(wk.A, tm.head, wk.Y, tm.s_head, wk.tickets, bt.status, st, act);
    k_tc_head_epi<<<ew, 256, 0, st>>>(m, bt, wk.Y, 1, tm.head.ntile * kTcBN);
    k_tc_stats<<<std::min(sms * 4, std::max(1, bt.B * nb / kPW)), kThreads, 0, st>>>(m, bt);
  }
  k_tc_finalize<<<bt.B, kThreads, 0, st>>>(bt);
  DEFER_CUDA(cudaGetLastError());
}

int launches_per_step_tc(const DModel& m) { return 5 + 11 * m.L; }

void tc_gemm_check(int device, const float* X, int M, const float* W, int N, int K, bool w_bf16, float* Y) {
  if (M < 1 || M > kTcM || N < 1 || K < 1) fail(kInvalidArgument, "tensor-core GEMM check: bad shape");
  DEFER_CUDA(cudaSetDevice(device));
  int sms = 0;
  DEFER_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  cudaStream_t st;
  DEFER_CUDA(cudaStreamCreate(&st));
  const size_t wbytes = (size_t)N * K * (w_bf16 ? 2 : 4);
  void *dW = nullptr, *dX = nullptr, *dP = nullptr, *dA = nullptr, *dY = nullptr, *dS = nullptr;
  DEFER_CUDA(cudaMalloc(&dW, wbytes));
  DEFER_CUDA(cudaMalloc(&dX, (size_t)M * K * 4));
  DEFER_CUDA(cudaMalloc(&dP, tc_packed_bytes(N, K, w_bf16)));
  DEFER_CUDA(cudaMalloc(&dA, tc_act_bytes(K)));
  DEFER_CUDA(cudaMalloc(&dS, sizeof(DSlotState) * M + 16));
  std::vector<DSlotState> sts(M);
  for (auto& z : sts) {
    memset(&z, 0, sizeof(z));
    z.active = 1;
  }
  if (w_bf16) {
    std::vector<uint16_t> wb((size_t)N * K);
    for (size_t i = 0; i < wb.size(); i++) {
      uint32_t u;
      memcpy(&u, &W[i], 4);
      wb[i] = (uint16_t)(u >> 16);  // the caller passes bf16-exact values
    }
    DEFER_CUDA(cudaMemcpy(dW, wb.data(), wbytes, cudaMemcpyHostToDevice));
  } else {
    DEFER_CUDA(cudaMemcpy(dW, W, wbytes, cudaMemcpyHostToDevice));
  }
  DEFER_CUDA(cudaMemcpy(dX, X, (size_t)M * K * 4, cudaMemcpyHostToDevice));
  DEFER_CUDA(cudaMemcpy(dS, sts.data(), sizeof(DSlotState) * M, cudaMemcpyHostToDevice));
  int* status = reinterpret_cast<int*>(static_cast<char*>(dS) + sizeof(DSlotState) * M);
  DEFER_CUDA(cudaMemset(status, 0, sizeof(int)));
  TcMatrix w = tc_pack(dW, N, K, w_bf16, static_cast<unsigned char*>(dP), st);
  const int splits = tc_splits(w, sms);
  void* dT = nullptr;
  DEFER_CUDA(cudaMalloc(&dY, tc_y_floats(w, splits) * sizeof(float)));
  DEFER_CUDA(cudaMalloc(&dT, (size_t)w.ntile * sizeof(unsigned)));
  DEFER_CUDA(cudaMemset(dT, 0, (size_t)w.ntile * sizeof(unsigned)));
  tc_prep(static_cast<float*>(dX), nullptr, 0.0f, K, M, static_cast<DSlotState*>(dS), static_cast<unsigned char*>(dA),
          tc_aterms(w), st);
  tc_gemm(static_cast<unsigned char*>(dA), w, static_cast<float*>(dY), splits, static_cast<unsigned*>(dT), status,
          st);
  const size_t n_pad = (size_t)w.ntile * kTcBN;
  std::vector<float> tot((size_t)kTcM * n_pad);  // the total, in split 0's rows
  std::vector<unsigned> tickets(w.ntile);
  int stat = 0;
  DEFER_CUDA(cudaMemcpyAsync(tot.data(), dY, tot.size() * 4, cudaMemcpyDeviceToHost, st));
  DEFER_CUDA(cudaMemcpyAsync(tickets.data(), dT, tickets.size() * sizeof(unsigned), cudaMemcpyDeviceToHost, st));
  DEFER_CUDA(cudaMemcpyAsync(&stat, status, sizeof(int), cudaMemcpyDeviceToHost, st));
  DEFER_CUDA(cudaStreamSynchronize(st));
  for (int r = 0; r < M; r++)
    for (int n = 0; n < N; n++) Y[(size_t)r * N + n] = tot[(size_t)r * n_pad + n];
  for (unsigned t : tickets)
    if (t != 0 && stat == kStOk) fail(kCuda, "tensor-core GEMM: a tile's split tickets were left non-zero");
  cudaFree(dT);
  cudaFree(dW);
  cudaFree(dX);
  cudaFree(dP);
  cudaFree(dA);
  cudaFree(dY);
  cudaFree(dS);
  cudaStreamDestroy(st);
  if (stat == kStTimeout) fail(kDeviceTimeout, "a bounded wait of the tensor-core GEMM timed out");
}

TcModel::~TcModel() {
  if (arena) cudaFree(arena);
  if (y_buf) cudaFree(y_buf);
  if (tickets) cudaFree(tickets);
}

TcModel* tc_model_build(const DModel& m, const std::vector<DLayer>& layers, int sms, cudaStream_t st) {
  const bool bf = m.bf16 != 0;
  std::unique_ptr<TcModel> t(new TcModel());
  size_t bytes = 0;
  for (int l = 0; l < m.L; l++)
    bytes += tc_packed_bytes(m.QKVR, m.H, bf) + tc_packed_bytes(m.H, m.QD, bf) + tc_packed_bytes(2 * m.FF, m.H, bf) +
             tc_packed_bytes(m.H, m.FF, bf);
  bytes += tc_packed_bytes(m.V, m.H, bf);
  const size_t act = tc_act_bytes(std::max({m.H, m.QD, m.FF}));
  DEFER_CUDA(cudaMalloc(&t->arena, bytes + act));
  t->bytes = bytes;
  t->max_act = act;
  unsigned char* p = static_cast<unsigned char*>(t->arena);
  auto pack = [&](const void* W, int N, int K) {
    TcMatrix w = tc_pack(W, N, K, bf, p, st);
    p += tc_packed_bytes(N, K, bf);
    return w;
  };
  t->layers.resize(m.L);
  for (int l = 0; l < m.L; l++) {
    TcLayer& T = t->layers[l];
    T.attn_norm = layers[l].attn_norm;
    T.ffn_norm = layers[l].ffn_norm;
    T.qkv = pack(layers[l].wqkv, m.QKVR, m.H);
    T.o = pack(layers[l].wo, m.H, m.QD);
    T.gu = pack(layers[l].wgu, 2 * m.FF, m.H);
    T.down = pack(layers[l].wdown, m.H, m.FF);
    T.s_qkv = tc_splits(T.qkv, sms);
    T.s_o = tc_splits(T.o, sms);
    T.s_gu = tc_splits(T.gu, sms);
    T.s_down = tc_splits(T.down, sms);
    t->max_y = std::max({t->max_y, tc_y_floats(T.qkv, T.s_qkv), tc_y_floats(T.o, T.s_o), tc_y_floats(T.gu, T.s_gu),
                         tc_y_floats(T.down, T.s_down)});
  }
  t->head = pack(m.head, m.V, m.H);
  t->s_head = tc_splits(t->head, sms);
  t->max_y = std::max(t->max_y, tc_y_floats(t->head, t->s_head));
  t->work.A = p;
  DEFER_CUDA(cudaMemsetAsync(t->work.A, 0, act, st));
  DEFER_CUDA(cudaMalloc(&t->y_buf, t->max_y * sizeof(float)));
  t->work.Y = t->y_buf;
  int max_tiles = t->head.ntile;
  for (const TcLayer& L : t->layers)
    max_tiles = std::max({max_tiles, L.qkv.ntile, L.o.ntile, L.gu.ntile, L.down.ntile});
  DEFER_CUDA(cudaMalloc(&t->tickets, (size_t)max_tiles * sizeof(unsigned)));
  DEFER_CUDA(cudaMemsetAsync(t->tickets, 0, (size_t)max_tiles * sizeof(unsigned), st));
  t->work.tickets = t->tickets;
  DEFER_CUDA(cudaStreamSynchronize(st));
  return t.release();
}

}  // namespace defer

// Phase functions of one token step (see device.cuh for the arithmetic
// contract). Included by kernels.cu (phase and grid-barrier kernels) and by
// flow.cu (dataflow kernel), each its own device module.
//
// A step is: SELECT (choose this step's token per slot, write the embedding
// row) | per layer: QKV (RMSNorm + projection + RoPE + KV append) | ATTN
// (chunk partials; the last chunk of each KV head combines) | O (+residual)
// | GATEUP (RMSNorm + gate/up + SiLU*up) | DOWN (+residual) | HEAD (final
// RMSNorm + lm_head + sampler block statistics) | for slots that sample at
// T > 0 next: SAMPLE1 (block e-sums) | SAMPLE2 (block p-sums). Each "|" is a
// grid-wide dependency (one barrier in the persistent kernel).
#pragma once
#include <cuda_runtime.h>

#include <climits>
#include <cstdint>

#include "device.cuh"

// CTA-wide barrier of the phase code. A kernel whose CTAs hold threads that
// do not run the phases (a weight-producer warp) defines it, before
// including this header, as a named barrier over the kThreads phase threads.
#ifndef DEFER_CTA_SYNC
#define DEFER_CTA_SYNC() __syncthreads()
#endif
// Threads that run the phase code in each CTA (a multiple of 32).
#ifndef DEFER_PHASE_THREADS
#define DEFER_PHASE_THREADS 256
#endif

namespace defer {

constexpr int kPT = DEFER_PHASE_THREADS;  // phase threads per CTA
constexpr int kPW = kPT / 32;             // phase warps per CTA

// ----------------------------------------------------------- primitives
// Weights never change while a kernel runs: streamed through the
// non-coherent path without allocating in L1.
__device__ __forceinline__ float4 ld_stream(const void* p) {
  float4 r;
  asm("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
      : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
      : "l"(p));
  return r;
}

__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

// Activations, KV entries and slot state are rewritten by other CTAs between
// phases of the persistent kernel, so they are read at L2 (ld.global.cg),
// never from a possibly stale L1 line or the non-coherent path.
__device__ __forceinline__ float4 ld_act(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float ld_f(const float* p) { return __ldcg(p); }
__device__ __forceinline__ int ld_i(const int* p) { return __ldcg(p); }
__device__ __forceinline__ uint32_t ld_u(const uint32_t* p) { return __ldcg(p); }

// Starts moving [p, p + bytes) from HBM into L2 without waiting (16-byte
// granules; p 16-byte aligned). Used to stream the next phase's weights
// while the current phase and its barrier run.
__device__ __forceinline__ void prefetch_l2(const void* p, size_t bytes) {
  const char* c = static_cast<const char*>(p);
  const size_t piece = 64 * 1024;
  for (size_t off = (size_t)(threadIdx.x & 31) * piece; off < bytes; off += 32 * piece) {
    const size_t n = (bytes - off < piece ? bytes - off : piece) & ~(size_t)15;
    if (n) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(c + off), "r"((unsigned)n) : "memory");
  }
}

__device__ __forceinline__ float warp_sum_butterfly(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// Max over the CTA's phase threads (every thread gets it). Whole CTA.
__device__ __forceinline__ float cta_max(float v) {
  __shared__ float s_w[kPW];
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) s_w[threadIdx.x >> 5] = v;
  DEFER_CTA_SYNC();
  float r = -INFINITY;
  for (int w = 0; w < kPW; w++) r = fmaxf(r, s_w[w]);
  DEFER_CTA_SYNC();
  return r;
}

// Sequential sum of the 32 lane values in lane order (all lanes get it).
__device__ __forceinline__ float warp_seq_sum(float v) {
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < 32; j++) s = __fadd_rn(s, __shfl_sync(0xffffffffu, v, j));
  return s;
}

__device__ __forceinline__ float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }

// Loads the 16-byte weight chunk j of a row as E fp32 values (exact).
template <bool BF16>
struct WChunk;
template <>
struct WChunk<false> {
  static constexpr int E = 4;
  // L1-allocating variant, for rows several warps of a CTA read in turn
  __device__ __forceinline__ static void load_l1(const void* row, int j, float* w) {
    const float4 t = __ldg(reinterpret_cast<const float4*>(row) + j);
    w[0] = t.x;
    w[1] = t.y;
    w[2] = t.z;
    w[3] = t.w;
  }
  __device__ __forceinline__ static void load(const void* row, int j, float* w) {
    float4 t = ld_stream(reinterpret_cast<const float4*>(row) + j);
    w[0] = t.x;
    w[1] = t.y;
    w[2] = t.z;
    w[3] = t.w;
  }
};
template <>
struct WChunk<true> {
  static constexpr int E = 8;
  __device__ __forceinline__ static void load_l1(const void* row, int j, float* w) {
    const uint4 t = __ldg(reinterpret_cast<const uint4*>(row) + j);
    w[0] = bf16_lo(t.x);
    w[1] = bf16_hi(t.x);
    w[2] = bf16_lo(t.y);
    w[3] = bf16_hi(t.y);
    w[4] = bf16_lo(t.z);
    w[5] = bf16_hi(t.z);
    w[6] = bf16_lo(t.w);
    w[7] = bf16_hi(t.w);
  }
  __device__ __forceinline__ static void load(const void* row, int j, float* w) {
    uint4 t = ld_stream_u4(reinterpret_cast<const uint4*>(row) + j);
    w[0] = bf16_lo(t.x);
    w[1] = bf16_hi(t.x);
    w[2] = bf16_lo(t.y);
    w[3] = bf16_hi(t.y);
    w[4] = bf16_lo(t.z);
    w[5] = bf16_hi(t.z);
    w[6] = bf16_lo(t.w);
    w[7] = bf16_hi(t.w);
  }
};

// Activation chunk of slot g: from shared memory (staged) or global (L2).
template <bool SMEM>
__device__ __forceinline__ float4 ld_x(const float* p) {
  if (SMEM) return *reinterpret_cast<const float4*>(p);
  return ld_act(p);
}

// Canonical warp dot product of NR weight rows against G activation
// vectors x_g = xs + g * xstride (all lanes return the same sums).
template <bool BF16, bool SMEM, int NR, int G, bool WSMEM = false>
__device__ __forceinline__ void warp_dot(const void* const (&rows)[NR], int K, const float* xs, int xstride,
                                         float (&acc)[NR][G]) {
  constexpr int E = WChunk<BF16>::E;
  const int lane = threadIdx.x & 31;
  const int nch = K / E;
#pragma unroll
  for (int r = 0; r < NR; r++)
#pragma unroll
    for (int g = 0; g < G; g++) acc[r][g] = 0.0f;
  // wide slot groups keep one chunk in flight (registers)
#pragma unroll(G <= 8 ? 4 : 1)
  for (int j = lane; j < nch; j += 32) {
    float w[NR][E];
#pragma unroll
    for (int r = 0; r < NR; r++) {
      if constexpr (WSMEM) {  // weight rows staged in shared memory
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
      } else {
        WChunk<BF16>::load(rows[r], j, w[r]);
      }
    }
#pragma unroll
    for (int g = 0; g < G; g++) {
      float xv[E];
#pragma unroll
      for (int q = 0; q < E / 4; q++) {
        float4 t = ld_x<SMEM>(xs + (size_t)g * xstride + j * E + 4 * q);
        xv[4 * q] = t.x;
        xv[4 * q + 1] = t.y;
        xv[4 * q + 2] = t.z;
        xv[4 * q + 3] = t.w;
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

// Register-tiled canonical dot of NR weight rows (row r at w0 + min(r, rmax)
// * wstride bytes; global memory, or shared memory when WSMEM) against NS
// activation vectors xs + s * xstride (shared memory when XSMEM, else
// global): the same per-lane chunk sums
// as warp_dot, but one warp carries all NR * NS = N (a power of two, >= 32)
// sums at once, so each chunk of x feeds NR rows and each chunk of W feeds
// NS slots. The cross-lane sum is a transpose reduction: at the level of
// lane distance d a lane keeps half of its sums and adds the partner's
// copy of the same half. Every sum is formed over the same pairs of lanes,
// in the same order, as warp_sum_butterfly, so the result is bit-identical;
// it needs N - N/32 shuffles instead of 5 N. Lane L ends holding the sums
// k = L * (N/32) + i (k = s * NR + r) as res[i], i < N/32.
//
// With NORM, x_s holds raw rows and every element is normalized as it is
// loaded, n = (x * inv[s]) * nw[i] (the RMSNorm of ops.rs:84-95, the same
// products as a staged normalized row).
template <bool BF16, bool WSMEM, bool XSMEM, int NR, int NS, bool NORM = false>
__device__ __forceinline__ void warp_tile(const unsigned char* w0, size_t wstride, int rmax, int K, const float* xs,
                                          int xstride, float (&res)[NR * NS / 32], const float* nw = nullptr,
                                          const float* inv = nullptr) {
  constexpr int E = WChunk<BF16>::E;
  constexpr int N = NR * NS;
  static_assert(N >= 32 && (N & (N - 1)) == 0, "tile must be a power of two of at least 32 sums");
  const int lane = threadIdx.x & 31;
  const int nch = K / E;
  float acc[N];
#pragma unroll
  for (int k = 0; k < N; k++) acc[k] = 0.0f;
  float sinv[NORM ? NS : 1];
  if constexpr (NORM) {
#pragma unroll
    for (int s = 0; s < NS; s++) sinv[s] = inv[s];
  }
  for (int j = lane; j < nch; j += 32) {
    float wn[NORM ? E : 1];
    if constexpr (NORM) {
#pragma unroll
      for (int q = 0; q < E / 4; q++) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(nw + j * E) + q);
        wn[4 * q] = t.x;
        wn[4 * q + 1] = t.y;
        wn[4 * q + 2] = t.z;
        wn[4 * q + 3] = t.w;
      }
    }
    float w[NR][E];
#pragma unroll
    for (int r = 0; r < NR; r++) {
      const unsigned char* row = w0 + (size_t)(r < rmax ? r : rmax) * wstride;
      if constexpr (WSMEM) {
        if constexpr (BF16) {
          const uint4 t = reinterpret_cast<const uint4*>(row)[j];
          w[r][0] = bf16_lo(t.x);
          w[r][1] = bf16_hi(t.x);
          w[r][2] = bf16_lo(t.y);
          w[r][3] = bf16_hi(t.y);
          w[r][4] = bf16_lo(t.z);
          w[r][5] = bf16_hi(t.z);
          w[r][6] = bf16_lo(t.w);
          w[r][7] = bf16_hi(t.w);
        } else {
          const float4 t = reinterpret_cast<const float4*>(row)[j];
          w[r][0] = t.x;
          w[r][1] = t.y;
          w[r][2] = t.z;
          w[r][3] = t.w;
        }
      } else {
        WChunk<BF16>::load_l1(row, j, w[r]);
      }
    }
#pragma unroll
    for (int s = 0; s < NS; s++) {
      float xv[E];
#pragma unroll
      for (int q = 0; q < E / 4; q++) {
        const float4 t = ld_x<XSMEM>(xs + (size_t)s * xstride + j * E + 4 * q);
        xv[4 * q] = t.x;
        xv[4 * q + 1] = t.y;
        xv[4 * q + 2] = t.z;
        xv[4 * q + 3] = t.w;
      }
      if constexpr (NORM) {
#pragma unroll
        for (int e = 0; e < E; e++) xv[e] = __fmul_rn(__fmul_rn(xv[e], sinv[s]), wn[e]);
      }
#pragma unroll
      for (int r = 0; r < NR; r++)
#pragma unroll
        for (int e = 0; e < E; e++) acc[s * NR + r] = fmaf(w[r][e], xv[e], acc[s * NR + r]);
    }
  }
  // transpose reduction, lane distances 16, 8, 4, 2, 1 (the butterfly's order)
#pragma unroll
  for (int lv = 0; lv < 5; lv++) {
    const int d = 16 >> lv;
    const int n = N >> lv, h = n >> 1;
    const bool up = (lane & d) != 0;
#pragma unroll
    for (int k = 0; k < h; k++) {
      const float send = up ? acc[k] : acc[k + h];
      const float keep = up ? acc[k + h] : acc[k];
      acc[k] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, d));
    }
  }
#pragma unroll
  for (int i = 0; i < N / 32; i++) res[i] = acc[i];
}

__device__ __forceinline__ size_t row_bytes(int K, bool bf16) { return (size_t)K * (bf16 ? 2 : 4); }

// Contiguous share [u0, u1) of `units` for CTA `cta` of `ncta`.
__device__ __forceinline__ void cta_range(int units, int cta, int ncta, int& u0, int& u1) {
  u0 = (int)((long long)units * cta / ncta);
  u1 = (int)((long long)units * (cta + 1) / ncta);
}

// Prefetch of this CTA's rows [u0*rows_per_unit, u1*rows_per_unit) of a
// matrix with K columns, when the whole matrix is small enough to sit in
// L2 next to the phase in flight.
constexpr size_t kPrefetchMaxBytes = 48u << 20;
__device__ __forceinline__ void prefetch_rows(const void* W, int rows_total, int K, bool bf16, int units, int per_unit,
                                              int cta, int ncta) {
  const size_t rb = row_bytes(K, bf16);
  if ((size_t)rows_total * rb > kPrefetchMaxBytes) return;
  if (threadIdx.x >= 32) return;
  int u0, u1;
  cta_range(units, cta, ncta, u0, u1);
  if (u1 > u0)
    prefetch_l2(static_cast<const char*>(W) + (size_t)u0 * per_unit * rb, (size_t)(u1 - u0) * per_unit * rb);
}

// ------------------------------------------------------------ RMSNorm
// Per-group slot state of the stage in flight (load_slot_state): whether
// slot b0 + g feeds a token this step, its position and its sampling
// temperature; g_live marks the rows stage_rows copied.
static __shared__ int g_act[kMaxGroupWide];
static __shared__ int g_pos[kMaxGroupWide];
static __shared__ float g_temp[kMaxGroupWide];
static __shared__ int g_live[kMaxGroupWide];

template <int G>
__device__ void load_slot_state(const DBatch& bt, int b0) {
  if (threadIdx.x < G) {
    const int b = b0 + threadIdx.x;
    g_act[threadIdx.x] = b < bt.B ? ld_i(&bt.st[b].active) : 0;
    g_pos[threadIdx.x] = b < bt.B ? ld_i(&bt.st[b].pos) : 0;
    g_temp[threadIdx.x] = b < bt.B ? bt.sess[b].temperature : 0.0f;
  }
  DEFER_CTA_SYNC();
}

__device__ __forceinline__ void cp_async16_g2s(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_prior1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Slot b0 + g's activations src[(b0 + g) * K + i] into dst[g * K + i] with
// cp.async (every copy in flight at once, no registers); slots past the
// batch, or inactive ones when `need_active`, become zeros. Also records the
// group's slot state in g_live / g_pos.
template <int G>
__device__ void stage_rows(const DBatch& bt, int b0, const float* src, int K, float* dst, bool need_active) {
  load_slot_state<G>(bt, b0);
  if (threadIdx.x < G) g_live[threadIdx.x] = b0 + (int)threadIdx.x < bt.B && (!need_active || g_act[threadIdx.x]);
  DEFER_CTA_SYNC();
  const int n4 = G * K / 4;  // K % 4 == 0
  // every CTA copies the same rows: each starts at its own offset so that
  // they do not all request the same L2 lines at the same moment
  const int rot = (int)((blockIdx.x * 32u) % (unsigned)n4);
  for (int f0 = threadIdx.x; f0 < n4; f0 += kPT) {
    const int f = f0 + rot < n4 ? f0 + rot : f0 + rot - n4;
    const int g = (4 * f) / K;
    if (g_live[g])
      cp_async16_g2s(dst + 4 * (size_t)f, src + (size_t)b0 * K + 4 * (size_t)f);
    else
      *reinterpret_cast<float4*>(dst + 4 * (size_t)f) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  DEFER_CTA_SYNC();
}

// Per-slot RMSNorm factors inv = 1 / sqrt(sum(x^2) / n + eps) of the group
// (g_inv), ops.rs:84-95. The raw rows are staged first; a warp computes the
// sums of squares of its slots g = warp, warp + kPW, ... side by side, each
// with the canonical dot (lane-strided float4 chunks, fmaf in element order,
// butterfly). Missing or inactive slots are zero rows.
static __shared__ float g_inv[kMaxGroupWide];

template <int G>
__device__ void stage_rows_inv(const DModel& m, const DBatch& bt, int b0, const float* x, float* dst) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  stage_rows<G>(bt, b0, x, m.H, dst, true);
  constexpr int Q = (G + kPW - 1) / kPW;
  float acc[Q];
#pragma unroll
  for (int q = 0; q < Q; q++) acc[q] = 0.0f;
  for (int j = lane; j < m.H / 4; j += 32) {
#pragma unroll
    for (int q = 0; q < Q; q++) {
      const int g = warp + q * kPW;
      if (g < G) {
        const float4 t = reinterpret_cast<const float4*>(dst + (size_t)g * m.H)[j];
        acc[q] = fmaf(t.x, t.x, acc[q]);
        acc[q] = fmaf(t.y, t.y, acc[q]);
        acc[q] = fmaf(t.z, t.z, acc[q]);
        acc[q] = fmaf(t.w, t.w, acc[q]);
      }
    }
  }
#pragma unroll
  for (int q = 0; q < Q; q++) {
    const int g = warp + q * kPW;
    const float ss = warp_sum_butterfly(acc[q]);
    if (lane == 0 && g < G) g_inv[g] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)m.H), m.eps)));
  }
  DEFER_CTA_SYNC();
}

// Staged raw rows of a group -> normalised rows (x * inv) * w in place,
// four consecutive elements per thread (H % 4 == 0); missing or inactive
// slots stay zero rows.
template <int G>
__device__ void scale_rows(const DModel& m, const float* w_of_layer, float* dst) {
  const int n4 = G * m.H / 4;
  for (int f = threadIdx.x; f < n4; f += kPT) {
    const int g = (4 * f) / m.H, i = 4 * f - g * m.H;
    float4 x = reinterpret_cast<float4*>(dst)[f];
    if (g_live[g]) {
      const float4 w = __ldg(reinterpret_cast<const float4*>(w_of_layer + i));
      const float inv = g_inv[g];
      x.x = __fmul_rn(__fmul_rn(x.x, inv), w.x);
      x.y = __fmul_rn(__fmul_rn(x.y, inv), w.y);
      x.z = __fmul_rn(__fmul_rn(x.z, inv), w.z);
      x.w = __fmul_rn(__fmul_rn(x.w, inv), w.w);
    } else {
      x = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    reinterpret_cast<float4*>(dst)[f] = x;
  }
  DEFER_CTA_SYNC();
}

// dst[g][i] = rmsnorm(x of slot b0+g)[i] = (x * inv) * w for the G slots of
// a group (inactive or missing slots get zeros), scaled in place.
template <int G>
__device__ void stage_norm(const DModel& m, const DBatch& bt, int b0, const float* w_of_layer, const float* x,
                           float* dst) {
  stage_rows_inv<G>(m, bt, b0, x, dst);
  scale_rows<G>(m, w_of_layer, dst);
}

// Copies slot activations [b0, b0+G) (stride K) into shared memory.
template <int G>
static __device__ void stage_copy(const DBatch& bt, int b0, const float* src, int K, float* dst) {
  stage_rows<G>(bt, b0, src, K, dst, false);
}

// Starts copying this CTA's weight rows [row0, row0 + nrows) (rb bytes
// each, 16-byte multiples) of W into shared memory after the stage's first
// x_floats floats, with cp.async; the next stage_rows (or cp_async_join)
// waits for them. Returns the copy, or null when it does not fit (the rows
// are then read from global memory).
static __device__ const unsigned char* stage_weights(const void* W, int row0, int nrows, size_t rb, float* smem,
                                                     size_t x_floats, unsigned smem_bytes) {
  const size_t off = ((x_floats + 3) & ~(size_t)3) * sizeof(float);
  const size_t bytes = (size_t)nrows * rb;
  if (nrows <= 0 || off + bytes > smem_bytes) return nullptr;
  unsigned char* dst = reinterpret_cast<unsigned char*>(smem) + off;
  const unsigned char* src = static_cast<const unsigned char*>(W) + (size_t)row0 * rb;
  for (size_t c = threadIdx.x; c < bytes / 16; c += kPT) cp_async16_g2s(dst + 16 * c, src + 16 * c);
  return dst;
}

__device__ __forceinline__ void cp_async_join() {
  asm volatile("cp.async.wait_all;" ::: "memory");
  DEFER_CTA_SYNC();
}

// --------------------------------------------------------------- sampler
struct ValIdx {
  float v;
  int i;
};

// b better than a: valid (non-NaN), larger, or equal with a lower index.
__device__ __forceinline__ bool vi_better(ValIdx b, ValIdx a) {
  if (b.i == INT_MAX) return false;
  if (a.i == INT_MAX) return true;
  return b.v > a.v || (b.v == a.v && b.i < a.i);
}

__device__ __forceinline__ ValIdx vi_warp_best(ValIdx x) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    ValIdx o{__shfl_xor_sync(0xffffffffu, x.v, off), __shfl_xor_sync(0xffffffffu, x.i, off)};
    if (vi_better(o, x)) x = o;
  }
  return x;
}

// e of logit l (NaN s counts as 0, sampler.rs:56).
__device__ __forceinline__ float e_of(float l, float T, float M) {
  const float s = __fdiv_rn(l, T);
  return isnan(s) ? 0.0f : expf(__fsub_rn(s, M));
}

// Sum over the warp of exp(s - mr) (0 for NaN s or an empty row): with the
// row's max mr, the statistics that steer the exact sampler's walk (their
// rounding is free).
__device__ __forceinline__ float row_expsum(float s, bool valid, float mr) {
  float z = (valid && !isnan(s) && mr > -INFINITY) ? expf(__fsub_rn(s, mr)) : 0.0f;
  for (int off = 16; off > 0; off >>= 1) z += __shfl_xor_sync(0xffffffffu, z, off);
  return z;
}

// Warp statistics of one 32-element block held one value per lane
// (`valid` false past the vocabulary): raw argmax, max of s = l / T and,
// when T != 0, the sum of exp(s - max).
__device__ __forceinline__ void block_stats(float l, int idx, bool valid, float T, float* lmax, int* larg,
                                            float* smax, float* zsum) {
  ValIdx me{l, (valid && !isnan(l)) ? idx : INT_MAX};
  ValIdx best = vi_warp_best(me);
  float s = -INFINITY;
  if (valid && T != 0.0f) s = __fdiv_rn(l, T);
  const float mr = warp_max(s);  // fmaxf skips NaN
  const float z = T != 0.0f ? row_expsum(s, valid, mr) : 0.0f;
  if ((threadIdx.x & 31) == 0) {
    *lmax = best.v;
    *larg = best.i;
    *smax = mr;
    *zsum = z;
  }
}

// Greedy choice from the block statistics (exact).
static __device__ uint32_t argmax_from_blocks(const float* lmax, const int* larg, int nblk, bool global_src) {
  ValIdx best{NAN, INT_MAX};
  for (int k = threadIdx.x; k < nblk; k += kPT) {
    ValIdx c{global_src ? ld_f(lmax + k) : lmax[k], global_src ? ld_i(larg + k) : larg[k]};
    if (vi_better(c, best)) best = c;
  }
  best = vi_warp_best(best);
  __shared__ float s_v[kPW];
  __shared__ int s_i[kPW];
  __shared__ int s_res;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    s_v[warp] = best.v;
    s_i[warp] = best.i;
  }
  DEFER_CTA_SYNC();
  if (warp == 0) {
    ValIdx c = lane < kPW ? ValIdx{s_v[lane], s_i[lane]} : ValIdx{NAN, INT_MAX};
    c = vi_warp_best(c);
    if (lane == 0) s_res = c.i == INT_MAX ? 0 : c.i;
  }
  DEFER_CTA_SYNC();
  const uint32_t r = (uint32_t)s_res;
  DEFER_CTA_SYNC();
  return r;
}

// ------------------------------------------------------- exact sampler
// The reference sampler (sampler.rs:43-109) on one logits vector by one
// CTA, with the reference's own sequential fp32 sums reproduced exactly:
//   s_i = l_i / T, M = max s_i (NaN skipped), e_i = exp(s_i - M) (0 for NaN
//   s_i), Z = e_0 + e_1 + ... in index order (fp32), degenerate Z -> the
//   greedy argmax; p_i = e_i * (1 / Z); r = 24 high bits of the word * 2^-24;
//   C = p_i added in index order over p_i > 0, the first i with r < C wins,
//   else the last i with p_i > 0.
// Exactness in parallel. While the running sum S stays in one binade
// [2^e, 2^(e+1)), every fp32 addition S + v rounds to the grid u = 2^(e-23),
// so S advances by q u with q the integer nearest v / u (a tie goes to the
// even multiple, so it depends on the parity of S / u): an integer sum,
// until S reaches 2^(e+1). The values are cut into rows of 32 consecutive
// values and blocks of 32 rows. From approximate prefix
// sums every row gets a predicted binade and, under it, its integer
// increment for an even and for an odd incoming multiple; blocks compose
// their rows' increments when all share one binade. Warp 0 then walks the
// blocks in order with the exact S, 32 items at a time: each lane composes
// the increments of the items up to its own and checks that they run in
// S's binade and stay below the next power of two; S jumps to the last
// item before the first that fails, and that item is descended into
// (block -> rows -> values; a value is added in fp32). A prediction only
// decides how far S jumps, never its value, so the result equals the
// sequential sum bit for bit. (e_i uses CUDA's expf; the reference's libm
// may differ in the last bit of some e_i.)

__device__ __forceinline__ unsigned long long gtimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

constexpr int kNoBinade = INT_MIN;       // no prediction: the item is descended into
constexpr int kAnyBinade = INT_MIN + 1;  // all values zero: S unchanged in any binade
constexpr int kStashRows = 32;           // rows without a prediction kept in shared memory

__device__ __forceinline__ int binade_of(float s) { return ((__float_as_int(s) >> 23) & 0xFF) - 127; }
__device__ __forceinline__ float pow2f(int k) { return __int_as_float((k + 127) << 23); }  // -126 <= k <= 127
// Binade of a running sum in which the integer steps apply (u and 2^24 u
// normal numbers), else kNoBinade (S = 0, tiny, huge or not finite).
__device__ __forceinline__ int walk_binade(float s) {
  if (!(s > 0.0f) || !isfinite(s)) return kNoBinade;
  const int e = binade_of(s);
  return e >= -102 && e <= 100 ? e : kNoBinade;
}

// v_i of one exact pass: e_i (Z) or p_i = e_i * inv (CDF).
struct SampleVals {
  const float* lg;
  float T, M, inv;
  bool p;
  __device__ __forceinline__ float raw(int i) const { return ld_f(lg + i); }
  __device__ __forceinline__ float of(float l) const {
    const float e = e_of(l, T, M);
    return p ? __fmul_rn(e, inv) : e;
  }
  __device__ __forceinline__ float operator()(int i) const { return of(raw(i)); }
};

// v_i of one exact pass from values held in shared memory: base[i - i0]
// is logit i (a CTA's own logits rows).
struct SharedVals {
  const float* base;
  int i0;
  float T, M, inv;
  bool p;
  __device__ __forceinline__ float raw(int i) const { return base[i - i0]; }
  __device__ __forceinline__ float of(float l) const {
    const float e = e_of(l, T, M);
    return p ? __fmul_rn(e, inv) : e;
  }
};

// Shared memory of sample_exact (floats): per row its sum, prefix, binade
// and two increments; per block the same but the sum; the stashed rows;
// one [32][9] transposition tile per warp.
__host__ __device__ __forceinline__ size_t sample_exact_floats(int V) {
  const size_t R = (size_t)(V + 31) / 32, NB = (R + 31) / 32;
  return 5 * R + 4 * NB + 32 * (size_t)kStashRows + (size_t)kPW * 32 * 9 + 8;
}

// Increments of a run of values in binade e (multiples of u = 2^(e-23)):
// d0 for an even incoming multiple, d1 for an odd one; saturate at 2^26.
struct Incr {
  int d0, d1;
};
// Run a, then run b (one binade).
__device__ __forceinline__ Incr incr_then(Incr a, Incr b) {
  Incr c;
  c.d0 = min(a.d0 + ((a.d0 & 1) ? b.d1 : b.d0), 1 << 26);
  c.d1 = min(a.d1 + (((1 + a.d1) & 1) ? b.d1 : b.d0), 1 << 26);
  return c;
}
// One value v >= 0 in binade e: q = v / u rounded to nearest; a tie takes
// the even total.
__device__ __forceinline__ Incr value_incr(float v, int e, bool* tie) {
  const float x = __fmul_rn(v, pow2f(23 - e));  // exact: a power-of-two scale
  *tie = false;
  if (!(x < 33554432.0f)) return Incr{1 << 25, 1 << 25};  // leaves the binade (or NaN)
  const float f = floorf(x);
  const float fr = __fsub_rn(x, f);
  const int fl = (int)f;
  if (fr == 0.5f) {
    *tie = true;
    return Incr{fl + (fl & 1), fl + ((fl + 1) & 1)};
  }
  const int q = fl + (fr > 0.5f ? 1 : 0);
  return Incr{q, q};
}

// One level of the walk, by warp 0: lane j holds item j (its binade and
// increments). S advances over items j0, j0 + 1, ... < n while each item is
// all zeros or runs in S's binade, S stays below the next power of two and
// (searching) r >= S. Returns the first item that stops it (n if none),
// with S the exact sum before that item.
struct WalkPos {
  float S;
  int f;
};
static __device__ __forceinline__ WalkPos walk_level_call(float S, int j0, int n, int e, int d0, int d1, int find,
                                                       float r) {
  const int lane = threadIdx.x & 31;
  const bool in = lane >= j0 && lane < n;
  const int eS = walk_binade(S);
  const bool ok = e == kAnyBinade || (eS != kNoBinade && e == eS);
  Incr t = (in && ok && e != kAnyBinade) ? Incr{d0, d1} : Incr{0, 0};
  if (__all_sync(0xffffffffu, t.d0 == t.d1)) {  // no ties: a plain prefix sum
    int x = t.d0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, off);
      if (lane >= off) x = min(x + y, 1 << 26);
    }
    t.d0 = t.d1 = x;
  } else {
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const Incr o{__shfl_up_sync(0xffffffffu, t.d0, off), __shfl_up_sync(0xffffffffu, t.d1, off)};
      if (lane >= off) t = incr_then(o, t);
    }
  }
  float Sj = S;
  bool stop = !ok;
  if (eS != kNoBinade) {
    const int M = (int)__fmul_rn(S, pow2f(23 - eS));
    const int dd = (M & 1) ? t.d1 : t.d0;
    if (M + dd >= (1 << 24)) stop = true;
    else Sj = __fmul_rn((float)(M + dd), pow2f(eS - 23));
  }
  if (find && r < Sj) stop = true;
  const unsigned sm = __ballot_sync(0xffffffffu, in && stop);
  const int f = sm ? __ffs(sm) - 1 : n;
  const float Sb = __shfl_sync(0xffffffffu, Sj, f > 0 ? min(f, 32) - 1 : 0);
  return WalkPos{f > j0 ? Sb : S, f};
}
__device__ __forceinline__ int walk_level(float& S, int j0, int n, int e, Incr d, bool find, float r) {
  const WalkPos p = walk_level_call(S, j0, n, e, d.d0, d.d1, find ? 1 : 0, r);
  S = p.S;
  return p.f;
}

// One row value by value (v = this lane's value, base = index of lane 0):
// integer runs in S's binade, fp32 additions where they stop. True when the
// walk ends here (the CDF hit, or a sum that is no longer finite).
struct WalkVals {
  float S, P;
  int hit, end;
};
static __device__ __forceinline__ WalkVals walk_values_call(float S, float P, int hit, float v, int base, int find,
                                                         float r) {
  int j0 = 0;
  for (int round = 0; round <= 32; round++) {  // every round consumes a value
    const int eS = walk_binade(S);
    bool tie;
    const Incr d = eS != kNoBinade ? value_incr(v, eS, &tie) : Incr{0, 0};
    const int e = v == 0.0f ? kAnyBinade : (eS != kNoBinade ? eS : kNoBinade);
    const int f = walk_level(S, j0, 32, e, d, find != 0, r);
    if (f >= 32) return WalkVals{S, P, hit, 0};
    const float vf = __shfl_sync(0xffffffffu, v, f);
    const float Sp = S;
    S = __fadd_rn(S, vf);
    if (find && vf > 0.0f && r < S) return WalkVals{S, Sp, base + f, 1};
    if (!isfinite(S)) return WalkVals{S, P, hit, 1};
    j0 = f + 1;
  }
  return WalkVals{S, P, hit, 0};
}
__device__ __forceinline__ bool walk_values(float& S, float& P, int& hit, float v, int base, bool find, float r) {
  const WalkVals w = walk_values_call(S, P, hit, v, base, find ? 1 : 0, r);
  S = w.S;
  P = w.P;
  hit = w.hit;
  return w.end != 0;
}

// Predicted binade of a row whose running sum goes from about lo to about
// lo + rs, or kNoBinade (straddles a power of two, starts at 0, or leaves
// the range where the integer steps apply): a kNoBinade row is one the
// walk expects to enter value by value.
__device__ __forceinline__ int predict_binade(float lo, float rs) {
  const float hi = lo + rs;
  if (lo > 0.0f && isfinite(hi)) {
    const int el = binade_of(lo);
    if (el == binade_of(hi) && el >= -102 && el <= 100) return el;
  }
  return kNoBinade;
}

// Increments of the 32 rows row0, row0 + 1, ... (lane = row; rows >= R
// contribute nothing) under each lane's predicted binade e. The values
// arrive 8 columns at a time through the warp's [32][9] tile of shared
// memory (a load instruction covers 4 rows x 8 columns: whole 32-byte
// sectors), computed where they are loaded; then each lane adds its row's
// values in order, keeping the running parity that ties need, for an even
// and an odd incoming multiple. *e_out: e, or kAnyBinade for an all-zero
// row; a kNoBinade row's values go to stash_row when it is non-null. Warp.
template <class Src>
__device__ __forceinline__ void rows_incr(const Src& v, int n, int row0, int R, int e, float* tile, float* stash_row,
                                          int* e_out, int* d0, int* d1) {
  const int lane = threadIdx.x & 31;
  const float scale = e != kNoBinade ? pow2f(23 - e) : 0.0f;
  int a0 = 0, a1 = 0;  // increments for an even / odd incoming multiple
  bool nz = false;
  for (int c = 0; c < 4; c++) {
    float raw[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int i = (row0 + k * 4 + (lane >> 3)) * 32 + c * 8 + (lane & 7);
      raw[k] = i < n ? v.raw(i) : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int rr = k * 4 + (lane >> 3);
      const int i = (row0 + rr) * 32 + c * 8 + (lane & 7);
      tile[rr * 9 + (lane & 7)] = i < n ? v.of(raw[k]) : 0.0f;
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const float x = tile[lane * 9 + j];
      nz |= x != 0.0f;
      if (stash_row) stash_row[c * 8 + j] = x;
      if (e != kNoBinade) {
        const float y = __fmul_rn(x, scale);  // exact: a power-of-two scale
        if (!(y < 33554432.0f)) {  // leaves the binade (or not finite)
          a0 = a1 = 1 << 26;
        } else {
          const float f = floorf(y);
          const float fr = __fsub_rn(y, f);
          const int fl = (int)f;
          if (fr == 0.5f) {  // a tie goes to the even total
            a0 += fl + ((a0 + fl) & 1);
            a1 += fl + ((1 + a1 + fl) & 1);
          } else {
            const int q = fl + (fr > 0.5f ? 1 : 0);
            a0 += q;
            a1 += q;
          }
          a0 = min(a0, 1 << 26);
          a1 = min(a1, 1 << 26);
        }
      }
    }
    __syncwarp();
  }
  (void)R;
  *e_out = nz ? e : kAnyBinade;
  *d0 = nz ? a0 : 0;
  *d1 = nz ? a1 : 0;
}

// Block composition and the walk over the rows' records (re, rd0, rd1:
// binade and increments, the stash slot of a kNoBinade row in rd0, -1 when
// its values are not stashed): the sum or CDF search of exact_seq. be, bd0,
// bd1: [NB] scratch. Whole CTA. `marks`: one stamp when the walk ends.
template <class Src>
static __device__ float exact_walk(const Src& v, int n, bool find, float r, int* found, float* prev, float* at,
                                   const int* re, const int* rd0, const int* rd1, int* be, int* bd0, int* bd1,
                                   const float* stash, unsigned long long* marks, int* seg) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int R = (n + 31) / 32, NB = (R + 31) / 32;
  __shared__ float s_res, s_prev, s_at;
  __shared__ int s_found;
  // segments: within a block, the rows between rows without a prediction.
  // seg[2 row] = the increments d0 from the segment's first row through
  // this one, seg[2 row + 1] = their binade code (e + 128, 254 all zero,
  // 255 mixed) << 16 | (d1 - d0 + 32768). A walk entering a segment at its
  // first row crosses it with one uniform step instead of a warp scan.
  for (int b = warp; b < NB; b += kPW) {
    const int row = b * 32 + lane;
    const int e = row < R ? re[row] : kAnyBinade;
    const bool flag = e == kNoBinade;
    const unsigned fm = __ballot_sync(0xffffffffu, flag);
    const unsigned below = fm & ((1u << lane) - 1u);
    const int start = below ? 32 - __clz(below) : 0;
    const bool real = !flag && e != kAnyBinade;
    // binade of the segment's first row with a prediction, if any
    const unsigned rm = __ballot_sync(0xffffffffu, real) & ~((1u << start) - 1u);
    const int first = rm ? __ffs(rm) - 1 : 32;
    const int ef = __shfl_sync(0xffffffffu, e, first < 32 ? first : 0);
    const unsigned mm = __ballot_sync(0xffffffffu, real && e != ef);  // (a real row has first <= lane)
    const unsigned span = (lane == 31 ? 0xffffffffu : ((1u << (lane + 1)) - 1u)) & ~((1u << start) - 1u);
    const bool uniform = (mm & span) == 0u;
    Incr t = real ? Incr{rd0[row], rd1[row]} : Incr{0, 0};
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const Incr o{__shfl_up_sync(0xffffffffu, t.d0, off), __shfl_up_sync(0xffffffffu, t.d1, off)};
      if (lane >= off && lane - off >= start) t = incr_then(o, t);
    }
    if (row < R && !flag) {
      const int es = !uniform ? kNoBinade : (first < 32 && first <= lane) ? ef : kAnyBinade;
      const uint32_t code = es == kNoBinade ? 255u : es == kAnyBinade ? 254u : (uint32_t)(es + 128);
      const bool sat = t.d0 >= (1 << 25) || t.d1 >= (1 << 25);
      seg[2 * row] = sat ? (1 << 26) : t.d0;
      seg[2 * row + 1] = (int)((code << 16) | (uint32_t)((sat ? 0 : t.d1 - t.d0) + 32768));
    }
  }
  // blocks: the composed increments when every row is all zeros or runs in
  // one binade
  for (int b = warp; b < NB; b += kPW) {
    const int row = b * 32 + lane;
    const int e = row < R ? re[row] : kAnyBinade;
    int common = kAnyBinade;
    const unsigned some = __ballot_sync(0xffffffffu, e != kAnyBinade);
    if (some) {
      const int e0 = __shfl_sync(0xffffffffu, e, __ffs(some) - 1);
      common = __all_sync(0xffffffffu, e == kAnyBinade || e == e0) ? e0 : kNoBinade;
    }
    Incr d = (row < R && e != kAnyBinade && e != kNoBinade) ? Incr{rd0[row], rd1[row]} : Incr{0, 0};
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const Incr o{__shfl_up_sync(0xffffffffu, d.d0, off), __shfl_up_sync(0xffffffffu, d.d1, off)};
      if (lane >= off) d = incr_then(o, d);
    }
    if (lane == 31) {
      be[b] = common;
      bd0[b] = d.d0;
      bd1[b] = d.d1;
    }
  }
  DEFER_CTA_SYNC();
  if (warp == 0) {  // the walk; every lane keeps the exact S
    float S = 0.0f, P = 0.0f;
    int hit = -1;
    bool end = false;
    for (int c = 0; c < NB && !end; c += 32) {
      const int nb = min(32, NB - c);
      const int eb = lane < nb ? be[c + lane] : kAnyBinade;
      const Incr db = lane < nb ? Incr{bd0[c + lane], bd1[c + lane]} : Incr{0, 0};
      for (int jb = 0; jb < nb && !end;) {
        const int fb = walk_level(S, jb, nb, eb, db, find, r);
        if (fb >= nb) break;
        const int b = c + fb;  // into the block's rows
        const int nr = min(32, R - b * 32);
        const int er = lane < nr ? re[b * 32 + lane] : kAnyBinade;
        const Incr dr = lane < nr ? Incr{rd0[b * 32 + lane], rd1[b * 32 + lane]} : Incr{0, 0};
        const unsigned fmask = __ballot_sync(0xffffffffu, lane < nr && er == kNoBinade);
        for (int jr = 0; jr < nr && !end;) {
          if (jr == 0 || ((fmask >> (jr - 1)) & 1u)) {
            // at a segment's first row: its rows up to the next row without
            // a prediction in one step, when they run in S's binade
            const unsigned ahead = fmask & ~((1u << jr) - 1u);
            const int endr = ahead ? __ffs(ahead) - 1 : nr;
            bool stepped = endr == jr;  // an empty segment
            if (endr > jr) {
              const int k = b * 32 + endr - 1;
              const int w0 = seg[2 * k], w1 = seg[2 * k + 1];
              const uint32_t code = (uint32_t)w1 >> 16;
              const int eS = walk_binade(S);
              if (code == 254u) {
                stepped = true;  // all zeros
              } else if (code != 255u && eS != kNoBinade && (int)code - 128 == eS) {
                const int M = (int)__fmul_rn(S, pow2f(23 - eS));
                const int dd = (M & 1) ? w0 + (w1 & 0xFFFF) - 32768 : w0;
                if (M + dd < (1 << 24)) {
                  const float Sn = __fmul_rn((float)(M + dd), pow2f(eS - 23));
                  if (!(find && r < Sn)) {
                    S = Sn;
                    stepped = true;
                  }
                }
              }
            }
            if (stepped) {
              if (endr >= nr) break;
              const int row = b * 32 + endr;  // the row without a prediction, value by value
              const int slot = __shfl_sync(0xffffffffu, dr.d0, endr);
              const int i = row * 32 + lane;
              const float x = slot >= 0 ? stash[slot * 32 + lane] : (i < n ? v(i) : 0.0f);
              end = walk_values(S, P, hit, x, row * 32, find, r);
              jr = endr + 1;
              continue;
            }
          }
          const int fr = walk_level(S, jr, nr, er, dr, find, r);
          if (fr >= nr) break;
          const int row = b * 32 + fr;  // into the row's values
          const int e_row = __shfl_sync(0xffffffffu, er, fr);
          const int slot = __shfl_sync(0xffffffffu, dr.d0, fr);
          const int i = row * 32 + lane;
          const float x = (e_row == kNoBinade && slot >= 0) ? stash[slot * 32 + lane] : (i < n ? v(i) : 0.0f);
          end = walk_values(S, P, hit, x, row * 32, find, r);
          jr = fr + 1;
        }
        jb = fb + 1;
      }
    }
    if (lane == 0) {
      if (marks) marks[0] = gtimer_ns();
      s_res = S;
      s_found = hit;
      s_prev = P;
      s_at = S;
    }
  }
  DEFER_CTA_SYNC();
  const float res = s_res;
  if (found) *found = s_found;
  if (prev) *prev = s_prev;
  if (at) *at = s_at;
  DEFER_CTA_SYNC();
  return res;
}

// The sequential fp32 sum of v(0..n) (find = false), or the CDF search
// (find = true): the first i with v_i > 0 and r < S_{i+1}, reported with
// the CDF before and at it; S is returned either way (the total when not
// found). smem[0..R) holds the rows' sums on entry (they only steer the
// walk, so any rounding will do).
static __device__ float exact_seq(const SampleVals& v, int n, bool find, float r, int* found, float* prev,
                                  float* at, float* smem, unsigned long long* marks = nullptr) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int R = (n + 31) / 32, NB = (R + 31) / 32;
  float* rs = smem;                                // [R] row sums
  float* rp = rs + R;                              // [R] row prefix
  int* re = reinterpret_cast<int*>(rp + R);        // [R] row binade
  int* rd0 = re + R;                               // [R] (stash slot of an unpredicted row)
  int* rd1 = rd0 + R;                              // [R]
  int* be = rd1 + R;                               // [NB] block binade
  int* bd0 = be + NB;                              // [NB]
  int* bd1 = bd0 + NB;                             // [NB]
  float* bp = reinterpret_cast<float*>(bd1 + NB);  // [NB] block prefix
  float* stash = bp + NB;                          // [kStashRows][32]
  __shared__ int s_nstash;
  if (tid == 0) s_nstash = 0;
  // prefixes: rows inside their block (warp per block), then the blocks
  for (int b = warp; b < NB; b += kPW) {
    const int row = b * 32 + lane;
    const float x = row < R ? rs[row] : 0.0f;
    float inc = x;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const float o = __shfl_up_sync(0xffffffffu, inc, off);
      if (lane >= off) inc += o;
    }
    const float ex = __shfl_up_sync(0xffffffffu, inc, 1);
    if (row < R) rp[row] = lane ? ex : 0.0f;
    if (lane == 31) bp[b] = inc;
  }
  DEFER_CTA_SYNC();
  if (warp == 0) {
    float carry = 0.0f;
    for (int b0 = 0; b0 < NB; b0 += 32) {
      const int b = b0 + lane;
      const float x = b < NB ? bp[b] : 0.0f;
      float inc = x;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float o = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += o;
      }
      if (b < NB) bp[b] = carry + (inc - x);
      carry += __shfl_sync(0xffffffffu, inc, 31);
    }
  }
  DEFER_CTA_SYNC();
  for (int row = tid; row < R; row += kPT) rp[row] += bp[row >> 5];
  DEFER_CTA_SYNC();
  // rows: predicted binade and increments, a warp per block of 32 rows
  float* tile = stash + 32 * kStashRows + warp * (32 * 9);
  for (int b = warp; b < NB; b += kPW) {
    const int row = b * 32 + lane;
    const bool has = row < R;
    int e = has ? predict_binade(rp[row], rs[row]) : kNoBinade;
    int slot = -1;  // stash slot of a row the walk will likely cross
    if (has && e == kNoBinade) {
      slot = atomicAdd(&s_nstash, 1);
      if (slot >= kStashRows) slot = -1;
    }
    int d0, d1;
    rows_incr(v, n, b * 32, R, e, tile, slot >= 0 ? stash + slot * 32 : nullptr, &e, &d0, &d1);
    if (has) {
      re[row] = e;
      rd0[row] = e == kNoBinade ? slot : d0;
      rd1[row] = d1;
    }
  }
  DEFER_CTA_SYNC();
  if (marks && tid == 0) marks[0] = gtimer_ns();
  return exact_walk(v, n, find, r, found, prev, at, re, rd0, rd1, be, bd0, bd1, stash, marks ? marks + 1 : nullptr,
                    reinterpret_cast<int*>(rs));  // the row sums and prefixes are done with: [2R] segments
}

// Row sums of v (the walk's steering; any rounding) into smem[0..R).
static __device__ void row_sums(const SampleVals& v, int n, float* rs) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int R = (n + 31) / 32;
  constexpr int kU = 8;
  for (int r0 = warp; r0 < R; r0 += kPW * kU) {
    float raw[kU];
#pragma unroll
    for (int u = 0; u < kU; u++) {
      const int i = (r0 + u * kPW) * 32 + lane;
      raw[u] = i < n ? v.raw(i) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < kU; u++) {
      const int row = r0 + u * kPW;
      if (row >= R) break;
      float x = row * 32 + lane < n ? v.of(raw[u]) : 0.0f;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
      if (lane == 0) rs[row] = x;
    }
  }
  DEFER_CTA_SYNC();
}

// Argmax of the raw logits (NaN skipped, lowest index on ties; 0 when all
// are NaN), M = max of s = l / T (T > 0), and the last index with
// predicate p_i > 0 when `inv` is given (lastp). Whole CTA.
static __device__ void logits_scan(const float* lg, int V, float T, int* amax, float* M) {
  ValIdx best{NAN, INT_MAX};
  float m = -INFINITY;
  for (int i = threadIdx.x; i < V; i += kPT) {
    const float l = ld_f(lg + i);
    const ValIdx c{l, isnan(l) ? INT_MAX : i};
    if (vi_better(c, best)) best = c;
    if (T != 0.0f) m = fmaxf(m, __fdiv_rn(l, T));
  }
  best = vi_warp_best(best);
  m = warp_max(m);
  __shared__ float s_v[kPW], s_m[kPW];
  __shared__ int s_i[kPW];
  __shared__ int s_res;
  __shared__ float s_max;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    s_v[warp] = best.v;
    s_i[warp] = best.i;
    s_m[warp] = m;
  }
  DEFER_CTA_SYNC();
  if (warp == 0) {
    ValIdx c = lane < kPW ? ValIdx{s_v[lane], s_i[lane]} : ValIdx{NAN, INT_MAX};
    float mm = lane < kPW ? s_m[lane] : -INFINITY;
    c = vi_warp_best(c);
    mm = warp_max(mm);
    if (lane == 0) {
      s_res = c.i == INT_MAX ? 0 : c.i;
      s_max = mm;
    }
  }
  DEFER_CTA_SYNC();
  *amax = s_res;
  *M = s_max;
  DEFER_CTA_SYNC();
}

// Last index with p_i > 0 (sampler.rs:101-108), -1 when none. Whole CTA.
static __device__ int last_positive(const SampleVals& v, int V) {
  int last = -1;
  for (int i = threadIdx.x; i < V; i += kPT)
    if (v(i) > 0.0f) last = i;
  for (int off = 16; off > 0; off >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, off));
  __shared__ int s_l[kPW];
  __shared__ int s_last;
  if ((threadIdx.x & 31) == 0) s_l[threadIdx.x >> 5] = last;
  DEFER_CTA_SYNC();
  if (threadIdx.x == 0) {
    int r = -1;
    for (int w = 0; w < kPW; w++) r = max(r, s_l[w]);
    s_last = r;
  }
  DEFER_CTA_SYNC();
  const int r = s_last;
  DEFER_CTA_SYNC();
  return r;
}

// sampler::sample_token with the PRNG word already drawn. *margin = the
// distance of r to the nearer edge of the chosen token's CDF interval (0
// for greedy, NaN for the degenerate one-hot fallback). smem:
// sample_exact_floats(V) floats. Whole CTA. `m_given`: M = m_max is known
// (the max of s gathered from per-CTA statistics), so no scan finds it.
// `row_m`, `row_z`: per row of 32 logits the max of s and the sum of
// exp(s - max) (block_stats), which steer the walk in place of a pass of
// row sums. `marks` (instrumentation, or null): globaltimer stamps when
// each pass's rows and blocks are ready and when its walk ends (4 words).
static __device__ uint32_t sample_exact(const float* lg, int V, float T, uint32_t word, float* margin,
                                                    float* smem,
                                       bool m_given = false, float m_max = 0.0f, const float* row_m = nullptr,
                                       const float* row_z = nullptr, unsigned long long* marks = nullptr) {
  int amax = 0;
  float M = m_max;
  if (!m_given || T == 0.0f) logits_scan(lg, V, T, &amax, &M);
  if (T == 0.0f) {
    *margin = 0.0f;
    return (uint32_t)amax;
  }
  const SampleVals ve{lg, T, M, 0.0f, false};
  if (row_m) {  // rows' max of s and sum of exp(s - max), from the logits' producers
    for (int row = threadIdx.x; row < (V + 31) / 32; row += kPT) {
      const float z = ld_f(row_z + row);
      smem[row] = z > 0.0f ? z * expf(ld_f(row_m + row) - M) : 0.0f;
    }
    DEFER_CTA_SYNC();
  } else {
    row_sums(ve, V, smem);
  }
  const float Z = exact_seq(ve, V, false, 0.0f, nullptr, nullptr, nullptr, smem, marks);
  if (!(Z > 0.0f) || !isfinite(Z)) {
    float unused;
    if (m_given) logits_scan(lg, V, T, &amax, &unused);
    *margin = NAN;
    return (uint32_t)amax;
  }
  const float inv = __fdiv_rn(1.0f, Z);
  const SampleVals vp{lg, T, M, inv, true};
  // rows of p, roughly (the sum's walk reused the row sums' space)
  if (row_m) {
    for (int row = threadIdx.x; row < (V + 31) / 32; row += kPT) {
      const float z = ld_f(row_z + row);
      smem[row] = z > 0.0f ? z * expf(ld_f(row_m + row) - M) * inv : 0.0f;
    }
    DEFER_CTA_SYNC();
  } else {
    row_sums(vp, V, smem);
  }
  const float r = (float)(word >> 8) * (1.0f / 16777216.0f);
  int hit;
  float prev, at;
  const float total = exact_seq(vp, V, true, r, &hit, &prev, &at, smem, marks ? marks + 2 : nullptr);
  if (hit >= 0) {
    *margin = fminf(__fsub_rn(r, prev), __fsub_rn(at, r));
    return (uint32_t)hit;
  }
  const int last = last_positive(vp, V);
  *margin = __fsub_rn(r, total);
  return (uint32_t)(last < 0 ? 0 : last);
}

// Whole sampler on one logits vector by one CTA (the exact sampler above).
static __device__ uint32_t sample_cta(const float* lg, int V, float T, uint32_t word, float* margin, float* smem) {
  return sample_exact(lg, V, T, word, margin, smem);
}

// ----------------------------------------------------------- select / embed
// Advances the slots that fed a token in the previous step, picks the
// token of this step for every slot (prompt token, sample from the
// previous step's statistics, or verified replay of a recorded token) and
// writes its embedding row. CTA unit = slot.
template <bool BF16>
__device__ void ph_select(const DModel& m, const DBatch& bt, int run_step, int cta, int ncta, float* smem) {
  const int tid = threadIdx.x;
  if (cta == 0 && tid == 0) bt.any_active[(run_step + 1) & 1] = 0;
  __shared__ int s_go, s_step;
  __shared__ uint32_t s_tok;
  for (int b = cta; b < bt.B; b += ncta) {
    DSlotState* st = bt.st + b;
    const DSession& S = bt.sess[b];
    // Thread 0 owns the slot state; the decisions every thread branches on
    // travel through shared memory (never re-read from global memory).
    if (tid == 0) {
      if (st->was_active) {
        st->pos += S.lanes;
        st->step += S.lanes;
      }
      st->was_active = 0;
      st->active = 0;
      // a lane of a position-parallel replay still verifies the index after
      // the last one it fed
      const int vi = st->step - S.lanes + 1;
      const bool verify_left = S.lanes > 1 && st->step >= S.lanes && vi < S.n_total;
      if (st->step >= S.n_total && !verify_left) st->done = 1;
      s_go = !st->done;
      s_step = st->step;
    }
    DEFER_CTA_SYNC();
    if (!s_go) {
      DEFER_CTA_SYNC();
      continue;
    }
    const int s = s_step;        // index fed in this step (none when >= n_total)
    const int vi = s - S.lanes + 1;  // index chosen from this slot's previous logits (= s for one lane)
    const bool feed = s < S.n_total;
    uint32_t tok = feed ? S.tokens[s] : 0u;
    if ((S.lanes == 1 || s >= S.lanes) && vi >= S.n_prompt && vi < S.n_total) {
      const int k = vi - S.n_prompt;
      const float T = S.temperature;
      const int nb = bt.nblk;
      float margin = 0.0f;
      uint32_t smp;
      if (T == 0.0f) {
        smp = argmax_from_blocks(bt.ss.lmax + (size_t)b * nb, bt.ss.larg + (size_t)b * nb, nb, true);
      } else {
        // M from the rows' maxima of s (the head's block statistics), which
        // with the rows' exp-sums also steer the exact walk
        const float* sm = bt.ss.smax + (size_t)b * nb;
        float mx = -INFINITY;
        for (int j = tid; j < nb; j += kPT) mx = fmaxf(mx, ld_f(sm + j));
        mx = cta_max(mx);
        smp = sample_exact(bt.logits + (size_t)b * m.V, m.V, T, S.words[k], &margin, smem, true, mx, sm,
                           bt.ss.esum + (size_t)b * nb);
      }
      if (S.verify) {
        if (tid == 0 && smp != S.tokens[vi]) {
          st->div_step = vi;
          st->div_token = smp;
          st->done = 1;
        }
      } else {  // generate mode has one lane: vi == s
        tok = smp;
        if (tid == 0) S.tokens[s] = smp;
      }
      if (tid == 0 && S.margins) S.margins[k] = margin;
    }
    if (tid == 0) {
      s_tok = 0xFFFFFFFFu;
      if (!feed) st->done = 1;  // a lane's last verification: nothing to feed
      if (!st->done) {
        if (tok >= (uint32_t)m.V) {
          atomicExch(bt.status, kStBadToken);
          st->done = 1;
        } else if (st->pos >= m.max_seq || st->pos >= S.cap) {
          atomicExch(bt.status, kStContext);
          st->done = 1;
        } else {
          st->cur = tok;
          st->active = 1;
          st->was_active = 1;
          bt.any_active[run_step & 1] = 1;
          s_tok = tok;
          if (!S.verify && s >= S.n_prompt) {
            for (int i = 0; i < S.n_stop; i++)
              if (S.stop[i] == tok) st->done = 1;  // fed now, nothing after it
          }
        }
      }
    }
    DEFER_CTA_SYNC();
    const uint32_t t = s_tok;
    if (t != 0xFFFFFFFFu) {
      float* x = bt.x + (size_t)b * m.H;
      if (BF16) {
        const uint16_t* e = reinterpret_cast<const uint16_t*>(m.embed) + (size_t)t * m.H;
        for (int i = tid; i < m.H; i += kPT) x[i] = __uint_as_float((uint32_t)e[i] << 16);
      } else {
        const float* e = reinterpret_cast<const float*>(m.embed) + (size_t)t * m.H;
        for (int i = tid; i < m.H; i += kPT) x[i] = e[i];
      }
    }
    DEFER_CTA_SYNC();
  }
}

// Slots that fed in the last step of a run advance their position.
static __device__ void ph_finalize(const DBatch& bt, int cta, int ncta) {
  if (threadIdx.x != 0) return;
  for (int b = cta; b < bt.B; b += ncta) {
    DSlotState* st = bt.st + b;
    if (st->was_active) {
      st->pos += bt.sess[b].lanes;
      st->step += bt.sess[b].lanes;
    }
    st->was_active = 0;
    st->active = 0;
    if (st->step >= bt.sess[b].n_total) st->done = 1;
  }
}

// ----------------------------------------------------------------- GEMVs
// Register-tiled projections for wide slot groups (G >= 8): a warp task is
// a tile of NU row units x 8 slots (warp_tile). The CTA's units [u0, u1)
// are cut into blocks of NU from u0; a block that would run past the last
// unit of the matrix is shifted back (its first units, which belong to the
// block or CTA before, are computed again and not written), so every tile
// reads whole rows. The CTA stages the union of its blocks' rows, [s0, s1).
struct TileBlocks {
  int nblk;    // blocks of this CTA
  int s0, s1;  // units the blocks read
};

__device__ __forceinline__ TileBlocks tile_blocks(int u0, int u1, int units, int NU) {
  TileBlocks t;
  t.nblk = (u1 - u0 + NU - 1) / NU;
  t.s0 = min(u0, units - NU);
  t.s1 = min(u0 + NU * t.nblk, units);
  return t;
}

// CTA partitions of the wide projections: CTA `cta` belongs to partition
// cta % P, whose CTAs split every row of the matrix among them and take the
// slot groups P * k + partition. Each CTA then stages only its partition's
// slots (the activations every CTA re-reads shrink by P) while the weights
// are read once per partition.
struct Part {
  int first;  // first slot of the partition's first group
  int step;   // slots between its groups
  int ci;     // CTA index inside the partition
  int nci;    // CTAs of the partition
};

template <int G>
__device__ __forceinline__ Part part_of(const DBatch& bt, int cta, int ncta) {
  const int P = bt.parts > 1 ? bt.parts : 1;
  const int p = cta % P;
  return Part{p * G, P * G, cta / P, (ncta - p + P - 1) / P};
}

// Nominal first unit of block i (the units it writes are [ub, min(ub + NU,
// u1))) and the first unit it computes.
__device__ __forceinline__ void tile_block(int u0, int i, int units, int NU, int& ub, int& ua) {
  ub = u0 + NU * i;
  ua = min(ub, units - NU);
}

// Epilogue of QKV unit u (rows 2u, 2u+1) for slot b at position pos: bias,
// RoPE of the pair (i, i + HALF) of a Q or K head, store to q or the cache.
__device__ __forceinline__ void qkv_store(const DModel& m, const DLayer& Ly, const DBatch& bt, int l, int u, int b,
                                          int pos, float a, float c) {
  const int qh = m.QD / 2, kh = m.KVD / 2;
  int sect, h, i;
  if (u < qh) {
    sect = 0;
    h = u / m.HALF;
    i = u % m.HALF;
  } else if (u < qh + kh) {
    sect = 1;
    h = (u - qh) / m.HALF;
    i = (u - qh) % m.HALF;
  } else {
    sect = 2;
    h = (u - qh - kh) / m.HALF;
    i = (u - qh - kh) % m.HALF;
  }
  if (Ly.bqkv) {
    a = __fadd_rn(a, Ly.bqkv[2 * u]);
    c = __fadd_rn(c, Ly.bqkv[2 * u + 1]);
  }
  if (sect < 2) {
    const float cs = m.rope_cos[(size_t)pos * m.HALF + i];
    const float sn = m.rope_sin[(size_t)pos * m.HALF + i];
    const float a2 = __fsub_rn(__fmul_rn(a, cs), __fmul_rn(c, sn));
    const float c2 = __fadd_rn(__fmul_rn(c, cs), __fmul_rn(a, sn));
    a = a2;
    c = c2;
  }
  if (sect == 0) {
    float* q = bt.q + (size_t)b * m.QD + h * m.HD;
    q[i] = a;
    q[i + m.HALF] = c;
  } else {
    const DSession& S = bt.sess[b];
    float* dst = (sect == 1 ? S.kc : S.vc) + (((size_t)l * m.NKV + h) * S.cap + pos) * m.HD;
    dst[i] = a;
    dst[i + m.HALF] = c;
  }
}

// act(gate) * up (SiLU or tanh-GELU), ops.rs:120-134.
__device__ __forceinline__ float gate_act_mul(const DModel& m, float gate, float up) {
  float act;
  if (m.gelu) {
    const float C = 0.7978846f;
    const float x3 = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, gate), gate), gate);
    act = __fmul_rn(__fmul_rn(0.5f, gate), __fadd_rn(1.0f, tanhf(__fmul_rn(C, __fadd_rn(gate, x3)))));
  } else {
    act = __fdiv_rn(gate, __fadd_rn(1.0f, expf(-gate)));
  }
  return __fmul_rn(act, up);
}

// Pair projection (QKV or gate/up) of a wide slot group: tiles of 4 row
// pairs x 8 slots; lane L ends holding slot L / 4 of the group's sub-group
// and the pair (rows 2 (L % 4), 2 (L % 4) + 1) of its block.
template <bool BF16, int G, bool GU>
__device__ void ph_pairs_wide(const DModel& m, const DBatch& bt, int l, int cta, int ncta, float* smem) {
  const DLayer& Ly = m.layers[l];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = GU ? m.FF : m.QKVR / 2;
  const void* W = GU ? Ly.wgu : Ly.wqkv;
  const float* nw = GU ? Ly.ffn_norm : Ly.attn_norm;
  constexpr int NU = 4, NSUB = G / 8;
  const Part pt = part_of<G>(bt, cta, ncta);
  int u0, u1;
  cta_range(units, pt.ci, pt.nci, u0, u1);
  if (u0 >= u1) return;
  const TileBlocks tb = tile_blocks(u0, u1, units, NU);
  const size_t rb = row_bytes(m.H, BF16);
  const unsigned char* wsm =
      stage_weights(W, 2 * tb.s0, 2 * (tb.s1 - tb.s0), rb, smem, (size_t)G * m.H, bt.smem_bytes);
  const unsigned char* wg = static_cast<const unsigned char*>(W);
  // When the CTA's rows do not fit shared memory whole, they stream through
  // it: SB row blocks per step (8 warp tasks), two step buffers, the next
  // step's copy in flight while the current one is multiplied.
  const size_t xb = (((size_t)G * m.H + 3) & ~(size_t)3) * sizeof(float);
  const size_t blk_bytes = (size_t)2 * NU * rb;
  const int SB_max = kPW / NSUB > 0 ? kPW / NSUB : 1;
  const size_t room = bt.smem_bytes > xb ? bt.smem_bytes - xb : 0;
  const int SB = wsm ? 0 : (int)min((size_t)SB_max, room / (2 * blk_bytes));
  unsigned char* sbuf = reinterpret_cast<unsigned char*>(smem) + xb;
  auto epilogue = [&](int b0, int ub, int ua, int sub, const float (&res)[2]) {
    const int u = ua + (lane & 3), gg = sub * 8 + (lane >> 2), b = b0 + gg;
    if (u < ub || u >= u1 || !g_act[gg]) return;
    if (GU) bt.g[(size_t)b * m.FF + u] = gate_act_mul(m, res[0], res[1]);
    else qkv_store(m, Ly, bt, l, u, b, g_pos[gg], res[0], res[1]);
  };
  for (int b0 = pt.first; b0 < bt.B; b0 += pt.step) {
    stage_rows_inv<G>(m, bt, b0, bt.x, smem);
    scale_rows<G>(m, nw, smem);  // once per group: every row block of the CTA reads these rows
    if (SB > 0) {
      const int nsteps = (tb.nblk + SB - 1) / SB;
      auto issue = [&](int stp) {
        if (stp < nsteps) {
          unsigned char* dst = sbuf + (size_t)(stp & 1) * SB * blk_bytes;
          for (int k = 0; k < SB && stp * SB + k < tb.nblk; k++) {
            int ub, ua;
            tile_block(u0, stp * SB + k, units, NU, ub, ua);
            const unsigned char* src = wg + (size_t)2 * ua * rb;
            for (size_t c = threadIdx.x; c < blk_bytes / 16; c += kPT)
              cp_async16_g2s(dst + (size_t)k * blk_bytes + 16 * c, src + 16 * c);
          }
        }
        cp_async_commit();
      };
      issue(0);
      for (int stp = 0; stp < nsteps; stp++) {
        issue(stp + 1);
        cp_async_wait_prior1();
        DEFER_CTA_SYNC();
        const unsigned char* buf = sbuf + (size_t)(stp & 1) * SB * blk_bytes;
        for (int task = warp; task < SB * NSUB; task += kPW) {
          const int k = task / NSUB, sub = task % NSUB, blk = stp * SB + k;
          if (blk >= tb.nblk) continue;
          int ub, ua;
          tile_block(u0, blk, units, NU, ub, ua);
          float res[2];
          warp_tile<BF16, true, true, 8, 8>(buf + (size_t)k * blk_bytes, rb, 7, m.H, smem + (size_t)sub * 8 * m.H,
                                            m.H, res);
          epilogue(b0, ub, ua, sub, res);
        }
        DEFER_CTA_SYNC();  // the step's buffer is refilled two steps later
      }
      asm volatile("cp.async.wait_all;" ::: "memory");
      continue;
    }
    for (int task = warp; task < tb.nblk * NSUB; task += kPW) {
      const int blk = task / NSUB, sub = task % NSUB;
      int ub, ua;
      tile_block(u0, blk, units, NU, ub, ua);
      float res[2];
      const float* xs = smem + (size_t)sub * 8 * m.H;
      if (wsm) warp_tile<BF16, true, true, 8, 8>(wsm + (size_t)2 * (ua - tb.s0) * rb, rb, 7, m.H, xs, m.H, res);
      else warp_tile<BF16, false, true, 8, 8>(wg + (size_t)2 * ua * rb, rb, 7, m.H, xs, m.H, res);
      epilogue(b0, ub, ua, sub, res);
    }
    DEFER_CTA_SYNC();
  }
}

// x[b] += W x_in[b] for a wide slot group: tiles of 4 rows x 8 slots; lane
// L ends holding row L % 4 of its block for slot L / 4 of the sub-group.
template <bool BF16, int G>
__device__ void ph_residual_wide(const DModel& m, const DBatch& bt, const void* W, int K, const float* xin, int cta,
                                 int ncta, float* smem, size_t smem_floats) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int NSUB = G / 8;
  const int units = m.H;
  const Part pt = part_of<G>(bt, cta, ncta);
  int u0, u1;
  cta_range(units, pt.ci, pt.nci, u0, u1);
  if (u0 >= u1) return;
  const bool staged = (size_t)G * K <= smem_floats;
  // the down projection (inputs wider than the hidden state) on a CTA with
  // 16 or more rows uses 8-row tiles (lane L: rows 2 (L % 4), +1 of slot
  // L / 4): half the activation loads per FMA and half the tasks; fewer rows
  // or short inputs keep 4-row tiles (measured faster there)
  const bool rows8 = staged && K > m.H && u1 - u0 >= 16 && units >= 8;
  const int NU = rows8 ? 8 : 4;
  const TileBlocks tb = tile_blocks(u0, u1, units, NU);
  const size_t rb = row_bytes(K, BF16);
  const unsigned char* wsm =
      stage_weights(W, tb.s0, tb.s1 - tb.s0, rb, smem, staged ? (size_t)G * K : 0, bt.smem_bytes);
  const unsigned char* wg = static_cast<const unsigned char*>(W);
  for (int b0 = pt.first; b0 < bt.B; b0 += pt.step) {
    if (staged) {
      stage_copy<G>(bt, b0, xin, K, smem);
    } else {
      load_slot_state<G>(bt, b0);
      cp_async_join();  // the weight rows
    }
    for (int task = warp; task < tb.nblk * NSUB; task += kPW) {
      const int blk = task / NSUB, sub = task % NSUB;
      int ub, ua;
      tile_block(u0, blk, units, NU, ub, ua);
      const unsigned char* w0 = wsm ? wsm + (size_t)(ua - tb.s0) * rb : wg + (size_t)ua * rb;
      if (rows8) {
        float res2[2];
        const float* xs = smem + (size_t)sub * 8 * K;
        if (wsm) warp_tile<BF16, true, true, 8, 8>(w0, rb, 7, K, xs, K, res2);
        else warp_tile<BF16, false, true, 8, 8>(w0, rb, 7, K, xs, K, res2);
        const int gg = sub * 8 + (lane >> 2), b = b0 + gg;
        if (!g_act[gg]) continue;
#pragma unroll
        for (int i = 0; i < 2; i++) {
          const int r = ua + 2 * (lane & 3) + i;
          if (r < ub || r >= u1) continue;
          float* x = bt.x + (size_t)b * m.H + r;
          *x = __fadd_rn(ld_f(x), res2[i]);
        }
        continue;
      }
      float res[1];
      if (staged) {
        const float* xs = smem + (size_t)sub * 8 * K;
        if (wsm) warp_tile<BF16, true, true, 4, 8>(w0, rb, 3, K, xs, K, res);
        else warp_tile<BF16, false, true, 4, 8>(w0, rb, 3, K, xs, K, res);
      } else {
        const float* xs = xin + (size_t)(b0 + sub * 8) * K;
        if (wsm) warp_tile<BF16, true, false, 4, 8>(w0, rb, 3, K, xs, K, res);
        else warp_tile<BF16, false, false, 4, 8>(w0, rb, 3, K, xs, K, res);
      }
      const int r = ua + (lane & 3), gg = sub * 8 + (lane >> 2), b = b0 + gg;
      if (r < ub || r >= u1 || !g_act[gg]) continue;
      float* x = bt.x + (size_t)b * m.H + r;
      *x = __fadd_rn(ld_f(x), res[0]);
    }
    DEFER_CTA_SYNC();  // the group's slot state and staged rows are reused by the next group
  }
}

// QKV projection (RMSNorm staged in smem) + bias + RoPE + KV append.
// Unit = row pair (rows 2u, 2u+1 of the pair-interleaved wqkv).
template <bool BF16, int G>
__device__ void ph_qkv(const DModel& m, const DBatch& bt, int l, int cta, int ncta, float* smem) {
  const DLayer& Ly = m.layers[l];
  prefetch_rows(Ly.wo, m.H, m.QD, BF16, m.H, 1, cta, ncta);  // the O projection comes next
  if constexpr (G >= 8) {
    ph_pairs_wide<BF16, G, false>(m, bt, l, cta, ncta, smem);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = m.QKVR / 2;
  int u0, u1;
  cta_range(units, cta, ncta, u0, u1);
  if (u0 >= u1) return;
  const size_t rb = row_bytes(m.H, BF16);
  const unsigned char* wsm =
      stage_weights(Ly.wqkv, 2 * u0, 2 * (u1 - u0), rb, smem, (size_t)G * m.H, bt.smem_bytes);
  // a wide slot group is split into sub-groups of up to 8 slots; tasks
  // (row unit, sub-group) spread over the warps (same arithmetic per slot)
  constexpr int GS = G < 8 ? G : 8, NS = G / GS;
  for (int b0 = 0; b0 < bt.B; b0 += G) {
    stage_norm<G>(m, bt, b0, Ly.attn_norm, bt.x, smem);
    for (int task = warp; task < (u1 - u0) * NS; task += kPW) {
      const int u = u0 + task / NS, sub = task % NS;
      float acc[2][GS];
      if (wsm) {
        const void* rows[2] = {wsm + (size_t)(2 * (u - u0)) * rb, wsm + (size_t)(2 * (u - u0) + 1) * rb};
        warp_dot<BF16, true, 2, GS, true>(rows, m.H, smem + (size_t)sub * GS * m.H, m.H, acc);
      } else {
        const char* base = reinterpret_cast<const char*>(Ly.wqkv);
        const void* rows[2] = {base + (size_t)(2 * u) * rb, base + (size_t)(2 * u + 1) * rb};
        warp_dot<BF16, true, 2, GS>(rows, m.H, smem + (size_t)sub * GS * m.H, m.H, acc);
      }
#pragma unroll
      for (int g = 0; g < GS; g++) {
        const int gg = sub * GS + g, b = b0 + gg;
        if (lane != g || !g_act[gg]) continue;
        qkv_store(m, Ly, bt, l, u, b, g_pos[gg], acc[0][g], acc[1][g]);
      }
    }
    DEFER_CTA_SYNC();
  }
}

// x[b] += W x_in[b] (O projection, down projection). Unit = row.
template <bool BF16, int G>
__device__ void ph_residual_gemv(const DModel& m, const DBatch& bt, const void* W, int K, const float* xin,
                                 int cta, int ncta, float* smem, size_t smem_floats) {
  if constexpr (G >= 8) {
    ph_residual_wide<BF16, G>(m, bt, W, K, xin, cta, ncta, smem, smem_floats);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int u0, u1;
  cta_range(m.H, cta, ncta, u0, u1);
  if (u0 >= u1) return;
  const size_t rb = row_bytes(K, BF16);
  const bool staged = (size_t)G * K <= smem_floats;
  const unsigned char* wsm = stage_weights(W, u0, u1 - u0, rb, smem, staged ? (size_t)G * K : 0, bt.smem_bytes);
  // a wide slot group is split into sub-groups of up to 8 slots; tasks
  // (row unit, sub-group) spread over the warps (same arithmetic per slot)
  constexpr int GS = G < 8 ? G : 8, NS = G / GS;
  for (int b0 = 0; b0 < bt.B; b0 += G) {
    if (staged) {
      stage_copy<G>(bt, b0, xin, K, smem);
    } else {
      load_slot_state<G>(bt, b0);
      cp_async_join();  // the weight rows
    }
    for (int task = warp; task < (u1 - u0) * NS; task += kPW) {
      const int r = u0 + task / NS, sub = task % NS;
      float acc[1][GS];
      if (wsm) {
        const void* rows[1] = {wsm + (size_t)(r - u0) * rb};
        if (staged) warp_dot<BF16, true, 1, GS, true>(rows, K, smem + (size_t)sub * GS * K, K, acc);
        else warp_dot<BF16, false, 1, GS, true>(rows, K, xin + (size_t)(b0 + sub * GS) * K, K, acc);
      } else {
        const void* rows[1] = {reinterpret_cast<const char*>(W) + (size_t)r * rb};
        if (staged) warp_dot<BF16, true, 1, GS>(rows, K, smem + (size_t)sub * GS * K, K, acc);
        else warp_dot<BF16, false, 1, GS>(rows, K, xin + (size_t)(b0 + sub * GS) * K, K, acc);
      }
#pragma unroll
      for (int g = 0; g < GS; g++) {
        const int gg = sub * GS + g, b = b0 + gg;
        if (lane != g || !g_act[gg]) continue;
        float* x = bt.x + (size_t)b * m.H + r;
        *x = __fadd_rn(ld_f(x), acc[0][g]);
      }
    }
    DEFER_CTA_SYNC();  // the group's slot state and staged rows are reused by the next group
  }
}

// gate/up projection (RMSNorm staged) + activation * up. Unit = j.
template <bool BF16, int G>
__device__ void ph_gateup(const DModel& m, const DBatch& bt, int l, int cta, int ncta, float* smem) {
  const DLayer& Ly = m.layers[l];
  prefetch_rows(Ly.wdown, m.H, m.FF, BF16, m.H, 1, cta, ncta);  // the down projection comes next
  if constexpr (G >= 8) {
    ph_pairs_wide<BF16, G, true>(m, bt, l, cta, ncta, smem);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int u0, u1;
  cta_range(m.FF, cta, ncta, u0, u1);
  if (u0 >= u1) return;
  const size_t rb = row_bytes(m.H, BF16);
  const unsigned char* wsm = stage_weights(Ly.wgu, 2 * u0, 2 * (u1 - u0), rb, smem, (size_t)G * m.H, bt.smem_bytes);
  // a wide slot group is split into sub-groups of up to 8 slots; tasks
  // (row unit, sub-group) spread over the warps (same arithmetic per slot)
  constexpr int GS = G < 8 ? G : 8, NS = G / GS;
  for (int b0 = 0; b0 < bt.B; b0 += G) {
    stage_norm<G>(m, bt, b0, Ly.ffn_norm, bt.x, smem);
    for (int task = warp; task < (u1 - u0) * NS; task += kPW) {
      const int j = u0 + task / NS, sub = task % NS;
      float acc[2][GS];
      if (wsm) {
        const void* rows[2] = {wsm + (size_t)(2 * (j - u0)) * rb, wsm + (size_t)(2 * (j - u0) + 1) * rb};
        warp_dot<BF16, true, 2, GS, true>(rows, m.H, smem + (size_t)sub * GS * m.H, m.H, acc);
      } else {
        const char* base = reinterpret_cast<const char*>(Ly.wgu);
        const void* rows[2] = {base + (size_t)(2 * j) * rb, base + (size_t)(2 * j + 1) * rb};
        warp_dot<BF16, true, 2, GS>(rows, m.H, smem + (size_t)sub * GS * m.H, m.H, acc);
      }
#pragma unroll
      for (int g = 0; g < GS; g++) {
        const int gg = sub * GS + g, b = b0 + gg;
        if (lane != g || !g_act[gg]) continue;
        bt.g[(size_t)b * m.FF + j] = gate_act_mul(m, acc[0][g], acc[1][g]);
      }
    }
    DEFER_CTA_SYNC();
  }
}

// Final RMSNorm + lm_head + sampler block statistics for a wide slot group:
// a warp task is (vocabulary block of kSBlk rows, sub-group of 8 slots),
// four tiles of 8 rows x 8 slots; the tile sums pass through a per-warp
// [8 slots][kSBlk rows] buffer so that lane r holds row r of each slot.
// Used when the staged variant below does not fit.
template <bool BF16, int G>
__device__ void ph_head_wide_direct(const DModel& m, const DBatch& bt, const Part& pt, int u0, int u1, float* smem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = bt.nblk;
  constexpr int NSUB = G / 8;
  const size_t rb = row_bytes(m.H, BF16);
  float* tbuf = smem + (((size_t)G * m.H + 3) & ~(size_t)3) + (size_t)warp * 8 * kSBlk;
  const unsigned char* wg = static_cast<const unsigned char*>(m.head);
  for (int b0 = pt.first; b0 < bt.B; b0 += pt.step) {
    stage_rows_inv<G>(m, bt, b0, bt.x, smem);
    scale_rows<G>(m, m.norm, smem);
    for (int task = warp; task < (u1 - u0) * NSUB; task += kPW) {
      const int k = u0 + task / NSUB, sub = task % NSUB;
      const float* xs = smem + (size_t)sub * 8 * m.H;
#pragma unroll 1
      for (int t = 0; t < kSBlk / 8; t++) {
        const int r0 = min(k * kSBlk + 8 * t, m.V - 1);
        float res[2];
        warp_tile<BF16, false, true, 8, 8>(wg + (size_t)r0 * rb, rb, m.V - 1 - r0, m.H, xs, m.H, res);
        const int s = lane >> 2, r = 8 * t + 2 * (lane & 3);
        tbuf[s * kSBlk + r] = res[0];
        tbuf[s * kSBlk + r + 1] = res[1];
      }
      __syncwarp();
      const int i = k * kSBlk + lane;
      const bool valid = i < m.V;
#pragma unroll 1
      for (int s = 0; s < 8; s++) {
        const int gg = sub * 8 + s, b = b0 + gg;
        if (!g_act[gg]) continue;
        const float v = tbuf[s * kSBlk + lane];
        if (valid) bt.logits[(size_t)b * m.V + i] = v;
        const size_t o = (size_t)b * nb + k;
        block_stats(v, i, valid, bt.sess[b].temperature, bt.ss.lmax + o, bt.ss.larg + o, bt.ss.smax + o,
                    bt.ss.esum + o);
      }
      __syncwarp();
    }
    DEFER_CTA_SYNC();
  }
}

// Shared-memory floats of the staged wide head: raw rows of the group, the
// [G][kSBlk] block of sums, and two half blocks (kSBlk / 2 rows) of weights.
__device__ __host__ __forceinline__ size_t head_staged_floats(int G, int H, bool bf16) {
  const size_t rows = (((size_t)G * H + 3) & ~(size_t)3) + (size_t)G * kSBlk;
  return rows + 2 * ((size_t)(kSBlk / 2) * H * (bf16 ? 2 : 4) / 4);
}


// The staged wide head: the CTA walks its vocabulary blocks in half blocks
// of 16 rows, each copied into shared memory with cp.async while the
// previous half is multiplied (two buffers); the 8 warps take the 8 tiles
// (2 row tiles x 4 sub-groups of a 32-slot group) of a half, so every
// weight row crosses L2 once per group and CTA. After both halves the
// block's [G][32] sums give each slot's logits and block statistics.
template <bool BF16, int G>
__device__ void ph_head_wide(const DModel& m, const DBatch& bt, int cta, int ncta, float* smem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = bt.nblk;
  static_assert(kSBlk == 32, "head tiles cover a 32-row block");
  const Part pt = part_of<G>(bt, cta, ncta);
  int u0, u1;
  cta_range(nb, pt.ci, pt.nci, u0, u1);
  if (u0 >= u1) return;
  constexpr int NSUB = G / 8;
  constexpr int HALF = kSBlk / 2;
  constexpr int TILES = (HALF / 8) * NSUB;  // warp tasks of a half block
  if (m.V % kSBlk != 0 || head_staged_floats(G, m.H, BF16) * sizeof(float) > bt.smem_bytes) {
    ph_head_wide_direct<BF16, G>(m, bt, pt, u0, u1, smem);
    return;
  }
  const size_t rb = row_bytes(m.H, BF16);
  float* sums = smem + (((size_t)G * m.H + 3) & ~(size_t)3);  // [G][kSBlk]
  unsigned char* wbuf = reinterpret_cast<unsigned char*>(sums + (size_t)G * kSBlk);
  const size_t half_bytes = (size_t)HALF * rb;
  const unsigned char* wg = static_cast<const unsigned char*>(m.head);
  const int nh = 2 * (u1 - u0);  // half blocks of this CTA
  for (int b0 = pt.first; b0 < bt.B; b0 += pt.step) {
    stage_rows_inv<G>(m, bt, b0, bt.x, smem);
    scale_rows<G>(m, m.norm, smem);
    auto issue = [&](int h) {
      if (h < nh) {
        const unsigned char* src = wg + ((size_t)u0 * kSBlk + (size_t)h * HALF) * rb;
        unsigned char* dst = wbuf + (size_t)(h & 1) * half_bytes;
        for (size_t c = threadIdx.x; c < half_bytes / 16; c += kPT) cp_async16_g2s(dst + 16 * c, src + 16 * c);
      }
      cp_async_commit();
    };
    issue(0);
    for (int h = 0; h < nh; h++) {
      issue(h + 1);
      cp_async_wait_prior1();  // this thread's copies of half h have landed
      DEFER_CTA_SYNC();        // ... and every thread's
      const unsigned char* wh = wbuf + (size_t)(h & 1) * half_bytes;
      for (int task = warp; task < TILES; task += kPW) {
        const int t = task / NSUB, sub = task % NSUB;
        float res[2];
        warp_tile<BF16, true, true, 8, 8>(wh + (size_t)8 * t * rb, rb, 7, m.H, smem + (size_t)sub * 8 * m.H, m.H,
                                          res);
        const int s = lane >> 2, r = (h & 1) * HALF + 8 * t + 2 * (lane & 3);
        float* row = sums + (size_t)(sub * 8 + s) * kSBlk;
        row[r] = res[0];
        row[r + 1] = res[1];
      }
      DEFER_CTA_SYNC();  // the half's buffer is free again; after an odd half the block's sums are complete
      if (h & 1) {
        // logits and block statistics of the block: a warp's slots warp,
        // warp + kPW, ... with their reductions interleaved (max and
        // lowest-index argmax do not depend on the order of combination)
        const int k = u0 + h / 2;
        const int i = k * kSBlk + lane;
        constexpr int Q = (G + kPW - 1) / kPW;
        ValIdx best[Q];
        float smx[Q], sown[Q];
#pragma unroll
        for (int q = 0; q < Q; q++) {
          const int gg = warp + q * kPW;
          const bool on = gg < G && g_act[gg];
          const float v = on ? sums[(size_t)gg * kSBlk + lane] : 0.0f;
          if (on) bt.logits[(size_t)(b0 + gg) * m.V + i] = v;
          const float T = on ? g_temp[gg] : 0.0f;
          best[q] = ValIdx{v, !isnan(v) ? i : INT_MAX};
          smx[q] = (on && T != 0.0f) ? __fdiv_rn(v, T) : -INFINITY;
          sown[q] = smx[q];
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
          for (int q = 0; q < Q; q++) {
            const ValIdx o{__shfl_xor_sync(0xffffffffu, best[q].v, off), __shfl_xor_sync(0xffffffffu, best[q].i, off)};
            if (vi_better(o, best[q])) best[q] = o;
            smx[q] = fmaxf(smx[q], __shfl_xor_sync(0xffffffffu, smx[q], off));
          }
        }
#pragma unroll
        for (int q = 0; q < Q; q++) {
          const int gg = warp + q * kPW;
          const bool samp = gg < G && g_act[gg] && g_temp[gg] != 0.0f;  // warp-uniform
          const float z = samp ? row_expsum(sown[q], true, smx[q]) : 0.0f;
          if (lane == 0 && gg < G && g_act[gg]) {
            const size_t o = (size_t)(b0 + gg) * nb + k;
            bt.ss.lmax[o] = best[q].v;
            bt.ss.larg[o] = best[q].i;
            bt.ss.smax[o] = smx[q];
            bt.ss.esum[o] = z;
          }
        }
        // the sums are rewritten from the next half on, after its barrier
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    DEFER_CTA_SYNC();
  }
}

// Final RMSNorm + lm_head + sampler block statistics. Unit = block of
// kSBlk vocabulary rows; lane r of the unit's warp ends holding row r.
template <bool BF16, int G>
__device__ void ph_head(const DModel& m, const DBatch& bt, int cta, int ncta, float* smem) {
  prefetch_rows(m.layers[0].wqkv, m.QKVR, m.H, BF16, m.QKVR / 2, 2, cta, ncta);  // next step's first phase
  if constexpr (G >= 8) {
    ph_head_wide<BF16, G>(m, bt, cta, ncta, smem);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = bt.nblk;
  int u0, u1;
  cta_range(nb, cta, ncta, u0, u1);
  if (u0 >= u1) return;
  const size_t rb = row_bytes(m.H, BF16);
  // a wide slot group is split into sub-groups of up to 8 slots; tasks
  // (row unit, sub-group) spread over the warps (same arithmetic per slot)
  constexpr int GS = G < 8 ? G : 8, NS = G / GS;
  for (int b0 = 0; b0 < bt.B; b0 += G) {
    stage_norm<G>(m, bt, b0, m.norm, bt.x, smem);
    for (int task = warp; task < (u1 - u0) * NS; task += kPW) {
      const int k = u0 + task / NS, sub = task % NS;
      float mine[GS];
#pragma unroll
      for (int g = 0; g < GS; g++) mine[g] = NAN;
      for (int r = 0; r < kSBlk; r += 2) {
        const int row0 = min(k * kSBlk + r, m.V - 1), row1 = min(k * kSBlk + r + 1, m.V - 1);
        const void* rows[2] = {reinterpret_cast<const char*>(m.head) + (size_t)row0 * rb,
                               reinterpret_cast<const char*>(m.head) + (size_t)row1 * rb};
        float acc[2][GS];
        warp_dot<BF16, true, 2, GS>(rows, m.H, smem + (size_t)sub * GS * m.H, m.H, acc);
#pragma unroll
        for (int g = 0; g < GS; g++) {
          if (lane == r) mine[g] = acc[0][g];
          if (lane == r + 1) mine[g] = acc[1][g];
        }
      }
      const int i = k * kSBlk + lane;
      const bool valid = i < m.V;
#pragma unroll
      for (int g = 0; g < GS; g++) {
        const int gg = sub * GS + g, b = b0 + gg;
        if (!g_act[gg]) continue;
        if (valid) bt.logits[(size_t)b * m.V + i] = mine[g];
        const size_t o = (size_t)b * nb + k;
        block_stats(mine[g], i, valid, bt.sess[b].temperature, bt.ss.lmax + o, bt.ss.larg + o, bt.ss.smax + o,
                    bt.ss.esum + o);
      }
    }
    DEFER_CTA_SYNC();
  }
}

// A run whose first step samples takes its logits from the previous run;
// their block statistics are recomputed here before the first SELECT.
__device__ __forceinline__ bool samples_first(const DBatch& bt, int b) {
  const DSession& S = bt.sess[b];
  return S.n_prompt == 0 && S.n_total > 0;
}

__device__ __forceinline__ bool any_first(const DBatch& bt, bool need_temperature) {
  for (int b = 0; b < bt.B; b++)
    if (samples_first(bt, b) && (!need_temperature || bt.sess[b].temperature != 0.0f)) return true;
  return false;
}

// Block statistics of the resident logits of every slot whose run starts
// with a sampling step. Unit = block of kSBlk logits.
static __device__ void ph_restat(const DModel& m, const DBatch& bt, int cta, int ncta) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = bt.nblk;
  int u0, u1;
  cta_range(nb, cta, ncta, u0, u1);
  for (int b = 0; b < bt.B; b++) {
    if (!samples_first(bt, b)) continue;
    const float T = bt.sess[b].temperature;
    const float* lg = bt.logits + (size_t)b * m.V;
    for (int k = u0 + warp; k < u1; k += kPW) {
      const int i = k * kSBlk + lane;
      const bool valid = i < m.V;
      const size_t o = (size_t)b * nb + k;
      block_stats(valid ? ld_f(lg + i) : NAN, i, valid, T, bt.ss.lmax + o, bt.ss.larg + o, bt.ss.smax + o,
                    bt.ss.esum + o);
    }
  }
}

// ------------------------------------------------------------- attention
// Two stages. CHUNKS: unit = (slot, KV head, chunk of kAttnChunk key
// positions) on CTA u mod ncta; a CTA walks its units with the next unit's
// queries, K rows and V rows copied into shared memory (cp.async, two
// buffers) while the current one is computed, and writes the chunk's
// partials (max m, sum l, unnormalised output acc) for each query head of
// the KV head; a head with a single chunk writes its output acc / l
// directly (what the combine gives for one chunk, bit for bit). COMBINE
// (after a grid-wide dependency): a warp per (slot, query head) with two or
// more chunks merges the partials in chunk order.

// Floats of one unit buffer: queries [Gh][HD], K rows [kAttnChunk][HD + 4]
// (padded: threads of a warp read different rows at the same column), V
// rows [kAttnChunk][HD].
__host__ __device__ __forceinline__ size_t attn_buf_floats(int Gh, int HD) {
  return (size_t)Gh * HD + (size_t)kAttnChunk * (HD + 4) + (size_t)kAttnChunk * HD;
}

// The chunk stage's shared memory: per-slot fields cached once per stage
// (K, V and mask pointers, active, pos, cap), then per CTA part its scores
// [Gh][kAttnChunk], chunk sums [Gh] and nbuf unit buffers.
constexpr int kAttnMaxBuf = 4;  // unit buffers per part: up to kAttnMaxBuf - 1 units in flight
constexpr int kAttnSlotFloats = 9;
__host__ __device__ __forceinline__ size_t attn_slot_floats(int B) {
  return ((size_t)kAttnSlotFloats * B + 3) & ~(size_t)3;
}
__host__ __device__ __forceinline__ size_t attn_part_floats(int Gh, int HD, int nbuf) {
  return (((size_t)Gh * kAttnChunk + Gh + 3) & ~(size_t)3) + (size_t)nbuf * attn_buf_floats(Gh, HD);
}
__host__ __device__ __forceinline__ size_t attn_smem_floats(int B, int Gh, int HD, int parts, int nbuf) {
  return attn_slot_floats(B) + (size_t)parts * attn_part_floats(Gh, HD, nbuf);
}

// Barrier of one CTA part: the whole CTA, or (two parts) its own half
// through named barrier 1 + part.
__device__ __forceinline__ void attn_part_sync(int parts, int part) {
  if (parts == 1) {
    DEFER_CTA_SYNC();
  } else {
    asm volatile("bar.sync %0, %1;" ::"r"(1 + part), "r"(kPT / 2) : "memory");
  }
}

// CHUNKS stage. The CTA splits into two independent parts of kPW / 2 warps
// when two parts with two unit buffers each fit its shared memory (a unit's
// work is a few short dependent chains, so two units in flight side by side
// keep more warps busy than one unit at a time), else it works as one part.
// Part p of CTA c takes units v, v + V, ... with v = c * parts + p and V =
// ncta * parts, and walks them with the next units' copies in flight.
static __device__ void ph_attn_chunks(const DModel& m, const DBatch& bt, int l, int cta, int ncta, float* smem) {
  {  // the gate/up projection comes after the O projection
    const DLayer& Ly = m.layers[l];
    prefetch_rows(Ly.wgu, 2 * m.FF, m.H, m.bf16 != 0, m.FF, 2, cta, ncta);
  }
  const int Gh = m.NH / m.NKV, HD = m.HD;
  const int maxc = bt.max_chunks;
  const int per_slot = m.NKV * maxc;
  const int units = bt.B * per_slot;
  const float** s_kc = reinterpret_cast<const float**>(smem);  // 8-byte aligned: the dynamic area is
  const float** s_vc = s_kc + bt.B;
  const uint32_t** s_mask = reinterpret_cast<const uint32_t**>(s_vc + bt.B);
  int* s_act = reinterpret_cast<int*>(s_mask + bt.B);
  int* s_pos = s_act + bt.B;
  int* s_cap = s_pos + bt.B;
  for (int b = threadIdx.x; b < bt.B; b += kPT) {
    s_act[b] = ld_i(&bt.st[b].active);
    s_pos[b] = ld_i(&bt.st[b].pos);
    const DSession& S = bt.sess[b];
    s_kc[b] = S.kc;
    s_vc[b] = S.vc;
    s_mask[b] = S.mask;
    s_cap[b] = S.cap;
  }
  DEFER_CTA_SYNC();
  const size_t bfl = attn_buf_floats(Gh, HD);
  const size_t have = bt.smem_bytes / sizeof(float), slots = attn_slot_floats(bt.B);
  const size_t room = have > slots ? have - slots : 0;
  const int parts = room >= 2 * attn_part_floats(Gh, HD, 2) ? 2 : 1;
  const size_t per_part = room / parts;
  int NB = 2;
  while (NB < kAttnMaxBuf && attn_part_floats(Gh, HD, NB + 1) <= per_part) NB++;
  const int nthr = kPT / parts;
  const int part = threadIdx.x / nthr;
  const int tid = threadIdx.x - part * nthr, warp = tid >> 5, lane = tid & 31, nw = nthr / 32;
  float* sc = smem + slots + (size_t)part * attn_part_floats(Gh, HD, NB);  // [Gh][kAttnChunk]
  float* lsum = sc + Gh * kAttnChunk;                                        // [Gh]
  float* buf0 = sc + (((size_t)Gh * kAttnChunk + Gh + 3) & ~(size_t)3);
  const int vstep = ncta * parts;
  auto live = [&](int u) {
    const int b = u / per_slot, c = u % maxc;
    return s_act[b] && c <= s_pos[b] / kAttnChunk;
  };
  auto next = [&](int u) {
    for (u += vstep; u < units; u += vstep)
      if (live(u)) return u;
    return -1;
  };
  auto issue = [&](int u, float* buf) {
    if (u >= 0) {
      const int b = u / per_slot, rem = u % per_slot, kvh = rem / maxc, c = rem % maxc;
      const float* kc = s_kc[b];
      const float* vc = s_vc[b];
      const int t0 = c * kAttnChunk, tn = min(kAttnChunk, s_pos[b] + 1 - t0);
      const size_t base = ((size_t)l * m.NKV + kvh) * s_cap[b] + t0;
      const float* qsrc = bt.q + (size_t)b * m.QD + (size_t)kvh * Gh * HD;
      float* qs = buf;
      float* ks = qs + Gh * HD;
      float* vs = ks + kAttnChunk * (HD + 4);
      const int c4n = HD / 4;
      for (int f = tid; f < Gh * c4n; f += nthr) cp_async16_g2s(qs + 4 * f, qsrc + 4 * f);
      if (nthr % c4n == 0) {
        // a thread's 16-byte column c4 stays fixed; its row advances by nthr / c4n
        const int c4 = tid % c4n, dt = nthr / c4n;
        const float* kg = kc + base * HD + 4 * c4;
        const float* vg = vc + base * HD + 4 * c4;
        for (int tt = tid / c4n; tt < tn; tt += dt) {
          cp_async16_g2s(ks + (size_t)tt * (HD + 4) + 4 * c4, kg + (size_t)tt * HD);
          cp_async16_g2s(vs + (size_t)tt * HD + 4 * c4, vg + (size_t)tt * HD);
        }
      } else {
        for (int f = tid; f < tn * c4n; f += nthr) {
          const int tt = f / c4n, c4 = f - tt * c4n;
          cp_async16_g2s(ks + (size_t)tt * (HD + 4) + 4 * c4, kc + (base + tt) * HD + 4 * c4);
          cp_async16_g2s(vs + (size_t)tt * HD + 4 * c4, vc + (base + tt) * HD + 4 * c4);
        }
      }
    }
    cp_async_commit();
  };
  // The part's walk is taken twice: u_iss, NB - 1 units ahead, issues the
  // copies (group j holds the j-th unit, or nothing), u computes.
  const int v0 = cta * parts + part;
  int u = v0 < units ? (live(v0) ? v0 : next(v0)) : -1;
  int u_iss = u, n_iss = 0;
  auto issue_next = [&]() {
    issue(u_iss, buf0 + (size_t)(n_iss % NB) * bfl);
    n_iss++;
    if (u_iss >= 0) u_iss = next(u_iss);
  };
  for (int j = 0; j < NB - 1; j++) issue_next();
  for (int it = 0; u >= 0; it++) {
    issue_next();  // into the buffer unit it - 1 used
    // every group but the NB - 1 newest has landed: unit it's among them
    if (NB == 2) asm volatile("cp.async.wait_group 1;" ::: "memory");
    else if (NB == 3) asm volatile("cp.async.wait_group 2;" ::: "memory");
    else asm volatile("cp.async.wait_group 3;" ::: "memory");
    attn_part_sync(parts, part);
    const float* qs = buf0 + (size_t)(it % NB) * bfl;
    const float* ks = qs + Gh * HD;
    const float* vs = ks + kAttnChunk * (HD + 4);
    const int b = u / per_slot, rem = u % per_slot, kvh = rem / maxc, c = rem % maxc;
    const uint32_t* mask = s_mask[b];
    const int pos = s_pos[b], nch = pos / kAttnChunk + 1;
    const int t0 = c * kAttnChunk, tn = min(kAttnChunk, pos + 1 - t0);
    for (int idx = tid; idx < Gh * kAttnChunk; idx += nthr) {
      const int h = idx / kAttnChunk, tt = idx - h * kAttnChunk;
      float sv = -INFINITY;
      const int t = t0 + tt;
      const bool masked = mask && t < pos && ((mask[t >> 5] >> (t & 31)) & 1u);
      if (tt < tn && !masked) {
        const float* kr = ks + (size_t)tt * (HD + 4);
        const float* qr = qs + h * HD;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll 4
        for (int d = 0; d < HD; d += 4) {
          const float4 k4 = *reinterpret_cast<const float4*>(kr + d);
          const float4 q4 = *reinterpret_cast<const float4*>(qr + d);  // same address in the warp: broadcast
          a0 = fmaf(q4.x, k4.x, a0);
          a1 = fmaf(q4.y, k4.y, a1);
          a2 = fmaf(q4.z, k4.z, a2);
          a3 = fmaf(q4.w, k4.w, a3);
        }
        sv = __fmul_rn(__fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3)), m.scale);
      }
      sc[idx] = sv;
    }
    attn_part_sync(parts, part);
    float* part_b = bt.part + (size_t)b * m.NH * maxc * (HD + 2);
    for (int h = warp; h < Gh; h += nw) {
      float* row = sc + h * kAttnChunk;
      const float v0s = row[lane], v1s = row[lane + 32];
      const float mx = warp_max(fmaxf(v0s, v1s));
      const float e0 = (v0s == -INFINITY) ? 0.0f : expf(__fsub_rn(v0s, mx));
      const float e1 = (v1s == -INFINITY) ? 0.0f : expf(__fsub_rn(v1s, mx));
      row[lane] = e0;
      row[lane + 32] = e1;
      const float ls = warp_sum_butterfly(__fadd_rn(e0, e1));
      if (lane == 0) {
        lsum[h] = ls;
        if (nch > 1) {
          float* pp = part_b + ((size_t)(kvh * Gh + h) * maxc + c) * (HD + 2);
          pp[0] = mx;
          pp[1] = ls;
        }
      }
    }
    attn_part_sync(parts, part);
    for (int idx = tid; idx < Gh * HD; idx += nthr) {
      const int h = idx / HD, d = idx - h * HD;
      const float* e = sc + h * kAttnChunk;  // e = 0 past tn
      float acc = 0.0f;
      for (int t4 = 0; t4 < tn; t4 += 4) {
        const float4 e4 = *reinterpret_cast<const float4*>(e + t4);  // broadcast
        const float* vr = vs + (size_t)t4 * HD + d;
        acc = fmaf(e4.x, vr[0], acc);
        if (t4 + 1 < tn) acc = fmaf(e4.y, vr[HD], acc);
        if (t4 + 2 < tn) acc = fmaf(e4.z, vr[2 * HD], acc);
        if (t4 + 3 < tn) acc = fmaf(e4.w, vr[3 * HD], acc);
      }
      if (nch > 1) part_b[((size_t)(kvh * Gh + h) * maxc + c) * (HD + 2) + 2 + d] = acc;
      else bt.att[(size_t)b * m.QD + (size_t)(kvh * Gh + h) * HD + d] = __fdiv_rn(acc, lsum[h]);
    }
    attn_part_sync(parts, part);  // the buffer, the scores and the sums are reused
    u = next(u);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  DEFER_CTA_SYNC();  // both parts done before the CTA leaves the stage
}

// Merge of the chunk partials of every (slot, query head) with two or more
// chunks, in chunk order: M = max m_c; w_c = exp(m_c - M) (0 for m_c = -inf);
// L = sum w_c l_c, O = sum w_c acc_c (fmaf, chunk order); out = O / L.
static __device__ void ph_attn_combine(const DModel& m, const DBatch& bt, int cta, int ncta) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int HD = m.HD, row = HD + 2, maxc = bt.max_chunks;
  const int tasks = bt.B * m.NH;
  for (int t = cta * kPW + warp; t < tasks; t += ncta * kPW) {
    const int b = t / m.NH, h = t - b * m.NH;
    if (!ld_i(&bt.st[b].active)) continue;
    const int nch = ld_i(&bt.st[b].pos) / kAttnChunk + 1;
    if (nch == 1) continue;  // written by the chunk stage
    const float* p = bt.part + ((size_t)b * m.NH + h) * maxc * row;
    float M = -INFINITY;
    for (int c = lane; c < nch; c += 32) M = fmaxf(M, ld_f(p + (size_t)c * row));
    M = warp_max(M);
    for (int d0 = 0; d0 < HD; d0 += 32) {
      const int d = d0 + lane;
      float L = 0.0f, O = 0.0f;
#pragma unroll 4
      for (int c = 0; c < nch; c++) {
        const float mc = ld_f(p + (size_t)c * row), lc = ld_f(p + (size_t)c * row + 1);
        const float ac = d < HD ? ld_f(p + (size_t)c * row + 2 + d) : 0.0f;
        const float w = (mc == -INFINITY) ? 0.0f : expf(__fsub_rn(mc, M));
        L = fmaf(w, lc, L);
        O = fmaf(w, ac, O);
      }
      if (d < HD) bt.att[(size_t)b * m.QD + (size_t)h * HD + d] = __fdiv_rn(O, L);
    }
  }
}

}  // namespace defer

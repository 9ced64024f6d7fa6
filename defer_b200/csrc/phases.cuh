// Phase functions of one token step (see device.cuh for the arithmetic
// contract). Included by kernels.cu only.
#pragma once
#include <cuda_runtime.h>

#include <climits>
#include <cstdint>

#include "device.cuh"

namespace defer {

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

__device__ __forceinline__ float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }

// Loads the 16-byte weight chunk j of a row as E fp32 values (exact).
template <bool BF16>
struct WChunk;
template <>
struct WChunk<false> {
  static constexpr int E = 4;
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

// Canonical warp dot product of NR weight rows against G activation
// vectors (all lanes return the same sums).
template <bool BF16, int NR, int G>
__device__ __forceinline__ void warp_dot(const void* const (&rows)[NR], int K, const float* const (&xs)[G],
                                         float (&acc)[NR][G]) {
  constexpr int E = WChunk<BF16>::E;
  const int lane = threadIdx.x & 31;
  const int nch = K / E;
#pragma unroll
  for (int r = 0; r < NR; r++)
#pragma unroll
    for (int g = 0; g < G; g++) acc[r][g] = 0.0f;
#pragma unroll 2
  for (int j = lane; j < nch; j += 32) {
    float w[NR][E];
#pragma unroll
    for (int r = 0; r < NR; r++) WChunk<BF16>::load(rows[r], j, w[r]);
#pragma unroll
    for (int g = 0; g < G; g++) {
      float xv[E];
#pragma unroll
      for (int q = 0; q < E / 4; q++) {
        float4 t = ld_act(xs[g] + j * E + 4 * q);
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

__device__ __forceinline__ size_t row_bytes(int K, bool bf16) { return (size_t)K * (bf16 ? 2 : 4); }

// ----------------------------------------------------------- select / embed
__device__ uint32_t sample_cta(const float* logits, int V, float T, uint32_t word, float* margin, float* smem);

// Advances the slots that fed a token in the previous step, then picks the
// token of this step for every slot (prompt token, sample, or verified
// replay of a recorded token). CTA unit = slot.
__device__ void ph_select(const DModel& m, const DBatch& bt, int run_step, int cta, int ncta, float* smem) {
  const int tid = threadIdx.x;
  if (cta == 0 && tid == 0) bt.any_active[(run_step + 1) & 1] = 0;
  __shared__ int s_go;
  for (int b = cta; b < bt.B; b += ncta) {
    DSlotState* st = bt.st + b;
    const DSession& S = bt.sess[b];
    if (tid == 0) {
      if (st->was_active) {
        st->pos += 1;
        st->step += 1;
      }
      st->was_active = 0;
      st->active = 0;
      if (st->step >= S.n_total) st->done = 1;
      s_go = !st->done;
    }
    __syncthreads();
    if (!s_go) {
      __syncthreads();
      continue;
    }
    const int s = ld_i(&st->step);
    uint32_t tok;
    if (s < S.n_prompt) {
      tok = S.tokens[s];
    } else {
      const int k = s - S.n_prompt;
      const float T = S.temperature;
      float margin = 0.0f;
      uint32_t smp = sample_cta(bt.logits + (size_t)b * m.V, m.V, T, T == 0.0f ? 0u : S.words[k], &margin, smem);
      if (S.verify) {
        tok = S.tokens[s];
        if (tid == 0 && smp != tok) {
          st->div_step = s;
          st->div_token = smp;
          st->done = 1;
        }
      } else {
        tok = smp;
        if (tid == 0) S.tokens[s] = smp;
      }
      if (tid == 0 && S.margins) S.margins[k] = margin;
    }
    if (tid == 0 && !st->done) {
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
        if (!S.verify && s >= S.n_prompt) {
          for (int i = 0; i < S.n_stop; i++)
            if (S.stop[i] == tok) st->done = 1;  // fed now, nothing after it
        }
      }
    }
    __syncthreads();
  }
}

// Slots that fed in the last step of a run advance their position.
__device__ void ph_finalize(const DBatch& bt, int cta, int ncta) {
  if (threadIdx.x != 0) return;
  for (int b = cta; b < bt.B; b += ncta) {
    DSlotState* st = bt.st + b;
    if (st->was_active) {
      st->pos += 1;
      st->step += 1;
    }
    st->was_active = 0;
    st->active = 0;
    if (st->step >= bt.sess[b].n_total) st->done = 1;
  }
}

template <bool BF16>
__device__ void ph_embed(const DModel& m, const DBatch& bt, int cta, int ncta) {
  for (int b = cta; b < bt.B; b += ncta) {
    if (!ld_i(&bt.st[b].active)) continue;
    const uint32_t tok = ld_u(&bt.st[b].cur);
    float* x = bt.x + (size_t)b * m.H;
    if (BF16) {
      const uint16_t* e = reinterpret_cast<const uint16_t*>(m.embed) + (size_t)tok * m.H;
      for (int i = threadIdx.x; i < m.H; i += kThreads) x[i] = __uint_as_float((uint32_t)e[i] << 16);
    } else {
      const float* e = reinterpret_cast<const float*>(m.embed) + (size_t)tok * m.H;
      for (int i = threadIdx.x; i < m.H; i += kThreads) x[i] = e[i];
    }
  }
}

// xn = rmsnorm(x, w) per active slot. CTA unit = slot.
__device__ void ph_norm(const DModel& m, const DBatch& bt, const float* w, int cta, int ncta) {
  __shared__ float s_inv;
  for (int b = cta; b < bt.B; b += ncta) {
    if (!ld_i(&bt.st[b].active)) continue;
    const float* x = bt.x + (size_t)b * m.H;
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      float acc = 0.0f;
      for (int j = lane; j < m.H / 4; j += 32) {
        float4 t = ld_act(x + 4 * j);
        acc = fmaf(t.x, t.x, acc);
        acc = fmaf(t.y, t.y, acc);
        acc = fmaf(t.z, t.z, acc);
        acc = fmaf(t.w, t.w, acc);
      }
      acc = warp_sum_butterfly(acc);
      if (lane == 0) s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)m.H), m.eps)));
    }
    __syncthreads();
    const float inv = s_inv;
    float* xn = bt.xn + (size_t)b * m.H;
    for (int i = threadIdx.x; i < m.H; i += kThreads) xn[i] = __fmul_rn(__fmul_rn(ld_f(x + i), inv), w[i]);
    __syncthreads();
  }
}

// ----------------------------------------------------------------- GEMVs
// QKV projection + bias + RoPE + KV append. Warp unit = row pair
// (rows 2u, 2u+1 of the pair-interleaved wqkv).
template <bool BF16, int G>
__device__ void ph_qkv(const DModel& m, const DBatch& bt, int l, int cta, int ncta) {
  const DLayer& Ly = m.layers[l];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = m.QKVR / 2;
  const size_t rb = row_bytes(m.H, BF16);
  const int qh = m.QD / 2, kh = m.KVD / 2;
  for (int b0 = 0; b0 < bt.B; b0 += G) {
    const float* xs[G];
#pragma unroll
    for (int g = 0; g < G; g++) xs[g] = bt.xn + (size_t)(b0 + g < bt.B ? b0 + g : b0) * m.H;
    for (int u = cta * kWarps + warp; u < units; u += ncta * kWarps) {
      const char* base = reinterpret_cast<const char*>(Ly.wqkv);
      const void* rows[2] = {base + (size_t)(2 * u) * rb, base + (size_t)(2 * u + 1) * rb};
      float acc[2][G];
      warp_dot<BF16, 2, G>(rows, m.H, xs, acc);
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
#pragma unroll
      for (int g = 0; g < G; g++) {
        const int b = b0 + g;
        if (lane != g || b >= bt.B || !ld_i(&bt.st[b].active)) continue;
        float a = acc[0][g], c = acc[1][g];
        if (Ly.bqkv) {
          a = __fadd_rn(a, Ly.bqkv[2 * u]);
          c = __fadd_rn(c, Ly.bqkv[2 * u + 1]);
        }
        const int pos = ld_i(&bt.st[b].pos);
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
    }
  }
}

// x[b] += W x_in[b] (O projection and down projection). Warp unit = row.
template <bool BF16, int G>
__device__ void ph_residual_gemv(const DModel& m, const DBatch& bt, const void* W, int K, const float* xin,
                                 int xin_stride, int cta, int ncta) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t rb = row_bytes(K, BF16);
  for (int b0 = 0; b0 < bt.B; b0 += G) {
    const float* xs[G];
#pragma unroll
    for (int g = 0; g < G; g++) xs[g] = xin + (size_t)(b0 + g < bt.B ? b0 + g : b0) * xin_stride;
    for (int r = cta * kWarps + warp; r < m.H; r += ncta * kWarps) {
      const void* rows[1] = {reinterpret_cast<const char*>(W) + (size_t)r * rb};
      float acc[1][G];
      warp_dot<BF16, 1, G>(rows, K, xs, acc);
#pragma unroll
      for (int g = 0; g < G; g++) {
        const int b = b0 + g;
        if (lane != g || b >= bt.B || !ld_i(&bt.st[b].active)) continue;
        float* x = bt.x + (size_t)b * m.H + r;
        *x = __fadd_rn(ld_f(x), acc[0][g]);
      }
    }
  }
}

// gate/up projection + activation * up. Warp unit = j (rows 2j, 2j+1).
template <bool BF16, int G>
__device__ void ph_gateup(const DModel& m, const DBatch& bt, int l, int cta, int ncta) {
  const DLayer& Ly = m.layers[l];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t rb = row_bytes(m.H, BF16);
  for (int b0 = 0; b0 < bt.B; b0 += G) {
    const float* xs[G];
#pragma unroll
    for (int g = 0; g < G; g++) xs[g] = bt.xn + (size_t)(b0 + g < bt.B ? b0 + g : b0) * m.H;
    for (int j = cta * kWarps + warp; j < m.FF; j += ncta * kWarps) {
      const char* base = reinterpret_cast<const char*>(Ly.wgu);
      const void* rows[2] = {base + (size_t)(2 * j) * rb, base + (size_t)(2 * j + 1) * rb};
      float acc[2][G];
      warp_dot<BF16, 2, G>(rows, m.H, xs, acc);
#pragma unroll
      for (int g = 0; g < G; g++) {
        const int b = b0 + g;
        if (lane != g || b >= bt.B || !ld_i(&bt.st[b].active)) continue;
        const float gate = acc[0][g], up = acc[1][g];
        float act;
        if (m.gelu) {
          const float C = 0.7978846f;
          const float x3 = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, gate), gate), gate);
          act = __fmul_rn(__fmul_rn(0.5f, gate), __fadd_rn(1.0f, tanhf(__fmul_rn(C, __fadd_rn(gate, x3)))));
        } else {
          act = __fdiv_rn(gate, __fadd_rn(1.0f, expf(-gate)));
        }
        bt.g[(size_t)b * m.FF + j] = __fmul_rn(act, up);
      }
    }
  }
}

// logits[b] = head · xn[b]. Warp unit = vocabulary row.
template <bool BF16, int G>
__device__ void ph_head(const DModel& m, const DBatch& bt, int cta, int ncta) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t rb = row_bytes(m.H, BF16);
  for (int b0 = 0; b0 < bt.B; b0 += G) {
    const float* xs[G];
#pragma unroll
    for (int g = 0; g < G; g++) xs[g] = bt.xn + (size_t)(b0 + g < bt.B ? b0 + g : b0) * m.H;
    for (int r = cta * kWarps + warp; r < m.V; r += ncta * kWarps) {
      const void* rows[1] = {reinterpret_cast<const char*>(m.head) + (size_t)r * rb};
      float acc[1][G];
      warp_dot<BF16, 1, G>(rows, m.H, xs, acc);
#pragma unroll
      for (int g = 0; g < G; g++) {
        const int b = b0 + g;
        if (lane != g || b >= bt.B || !ld_i(&bt.st[b].active)) continue;
        bt.logits[(size_t)b * m.V + r] = acc[0][g];
      }
    }
  }
}

// ------------------------------------------------------------- attention
// Partial attention of one key chunk for the query heads of one KV head.
// CTA unit = (slot, kv head, chunk). smem: G*HD + G*kAttnChunk floats.
__device__ void ph_attn(const DModel& m, const DBatch& bt, int l, int cta, int ncta, float* smem) {
  const int G = m.NH / m.NKV;
  const int maxc = bt.max_chunks;
  const int units = bt.B * m.NKV * maxc;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* qs = smem;             // [G][HD]
  float* sc = smem + G * m.HD;  // [G][kAttnChunk]
  for (int u = cta; u < units; u += ncta) {
    const int b = u / (m.NKV * maxc);
    const int rem = u % (m.NKV * maxc);
    const int kvh = rem / maxc, c = rem % maxc;
    if (!ld_i(&bt.st[b].active)) continue;
    const int pos = ld_i(&bt.st[b].pos);
    if (c > pos / kAttnChunk) continue;
    const DSession& S = bt.sess[b];
    const int t0 = c * kAttnChunk;
    const int tn = min(kAttnChunk, pos + 1 - t0);
    const float* qsrc = bt.q + (size_t)b * m.QD + (size_t)kvh * G * m.HD;
    for (int i = tid; i < G * m.HD; i += kThreads) qs[i] = ld_f(qsrc + i);
    __syncthreads();
    const size_t head_base = ((size_t)l * m.NKV + kvh) * S.cap;
    const float* kb = S.kc + (head_base + t0) * m.HD;
    for (int idx = tid; idx < G * kAttnChunk; idx += kThreads) {
      const int h = idx / kAttnChunk, tt = idx % kAttnChunk;
      float s = -INFINITY;
      const int t = t0 + tt;
      const bool masked = S.mask && t < pos && ((S.mask[t >> 5] >> (t & 31)) & 1u);
      if (tt < tn && !masked) {
        const float* kr = kb + (size_t)tt * m.HD;
        const float* qr = qs + h * m.HD;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        for (int d = 0; d < m.HD; d += 4) {
          const float4 k4 = ld_act(kr + d);
          a0 = fmaf(qr[d], k4.x, a0);
          a1 = fmaf(qr[d + 1], k4.y, a1);
          a2 = fmaf(qr[d + 2], k4.z, a2);
          a3 = fmaf(qr[d + 3], k4.w, a3);
        }
        s = __fmul_rn(__fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3)), m.scale);
      }
      sc[idx] = s;
    }
    __syncthreads();
    float* part_b = bt.part + (size_t)b * m.NH * maxc * (m.HD + 2);
    for (int h = warp; h < G; h += kWarps) {
      float* row = sc + h * kAttnChunk;
      const float v0 = row[lane], v1 = row[lane + 32];
      const float mx = warp_max(fmaxf(v0, v1));
      const float e0 = (v0 == -INFINITY) ? 0.0f : expf(__fsub_rn(v0, mx));
      const float e1 = (v1 == -INFINITY) ? 0.0f : expf(__fsub_rn(v1, mx));
      row[lane] = e0;
      row[lane + 32] = e1;
      const float ls = warp_sum_butterfly(__fadd_rn(e0, e1));
      if (lane == 0) {
        float* p = part_b + ((size_t)(kvh * G + h) * maxc + c) * (m.HD + 2);
        p[0] = mx;
        p[1] = ls;
      }
    }
    __syncthreads();
    const float* vb = S.vc + (head_base + t0) * m.HD;
    for (int idx = tid; idx < G * m.HD; idx += kThreads) {
      const int h = idx / m.HD, d = idx % m.HD;
      const float* e = sc + h * kAttnChunk;
      float acc = 0.0f;
      for (int tt = 0; tt < tn; tt++) acc = fmaf(e[tt], ld_f(vb + (size_t)tt * m.HD + d), acc);
      part_b[((size_t)(kvh * G + h) * maxc + c) * (m.HD + 2) + 2 + d] = acc;
    }
    __syncthreads();
  }
}

// Combines the chunk partials of one query head in chunk order.
// CTA unit = (slot, head).
__device__ void ph_combine(const DModel& m, const DBatch& bt, int cta, int ncta) {
  const int maxc = bt.max_chunks;
  for (int u = cta; u < bt.B * m.NH; u += ncta) {
    const int b = u / m.NH, h = u % m.NH;
    if (!ld_i(&bt.st[b].active)) continue;
    const int nch = ld_i(&bt.st[b].pos) / kAttnChunk + 1;
    const float* p = bt.part + ((size_t)b * m.NH + h) * maxc * (m.HD + 2);
    const int d = threadIdx.x;
    if (d >= m.HD) continue;
    float M = -INFINITY;
    for (int c = 0; c < nch; c++) M = fmaxf(M, ld_f(p + (size_t)c * (m.HD + 2)));
    float L = 0.0f, O = 0.0f;
    for (int c = 0; c < nch; c++) {
      const float* pc = p + (size_t)c * (m.HD + 2);
      const float mc = ld_f(pc), lc = ld_f(pc + 1), ac = ld_f(pc + 2 + d);
      const float w = (mc == -INFINITY) ? 0.0f : expf(__fsub_rn(mc, M));
      L = fmaf(w, lc, L);
      O = fmaf(w, ac, O);
    }
    bt.att[(size_t)b * m.QD + h * m.HD + d] = __fdiv_rn(O, L);
  }
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

// argmax with the reference's rules (sampler.rs:24-40): NaN skipped,
// strict > so the lowest index wins ties, 0 when every value is NaN.
__device__ uint32_t argmax_cta(const float* l, int V, float* smem) {
  ValIdx best{NAN, INT_MAX};
  for (int i = threadIdx.x; i < V; i += kThreads) {
    const float v = ld_f(l + i);
    if (isnan(v)) continue;
    ValIdx c{v, i};
    if (vi_better(c, best)) best = c;
  }
  best = vi_warp_best(best);
  float* sv = smem;
  int* si = reinterpret_cast<int*>(smem + kWarps);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) {
    sv[warp] = best.v;
    si[warp] = best.i;
  }
  __syncthreads();
  ValIdx r{NAN, INT_MAX};
  if (warp == 0) {
    ValIdx c = lane < kWarps ? ValIdx{sv[lane], si[lane]} : ValIdx{NAN, INT_MAX};
    r = vi_warp_best(c);
  }
  __syncthreads();
  if (threadIdx.x == 0) si[0] = r.i == INT_MAX ? 0 : r.i;
  __syncthreads();
  const uint32_t out = (uint32_t)si[0];
  __syncthreads();
  return out;
}

__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = -INFINITY;
  for (int w = 0; w < kWarps; w++) r = fmaxf(r, red[w]);
  __syncthreads();
  return r;
}

__device__ __forceinline__ int block_max_int(int v, int* red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, off));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  int r = INT_MIN;
  for (int w = 0; w < kWarps; w++) r = max(r, red[w]);
  __syncthreads();
  return r;
}

// Unnormalised (e) or normalised (p = e * inv) probability of element i.
__device__ __forceinline__ float prob_at(const float* l, int V, int i, float T, float M, float inv, bool norm) {
  if (i >= V) return 0.0f;
  const float s = __fdiv_rn(ld_f(l + i), T);
  const float e = isnan(s) ? 0.0f : expf(__fsub_rn(s, M));
  return norm ? __fmul_rn(e, inv) : e;
}

// Sums of the 256-element blocks (8 per lane, sequential at each level).
__device__ void block_sums(const float* l, int V, float T, float M, float inv, bool norm, float* bsum, int nblk) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int k = warp; k < nblk; k += kWarps) {
    const int i0 = k * 256 + lane * 8;
    float ls = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; e++) ls = __fadd_rn(ls, prob_at(l, V, i0 + e, T, M, inv, norm));
    float bs = 0.0f;
    for (int j = 0; j < 32; j++) bs = __fadd_rn(bs, __shfl_sync(0xffffffffu, ls, j));
    if (lane == 0) bsum[k] = bs;
  }
}

// Temperature sampling (sampler.rs:43-109) with the canonical hierarchical
// sums. Returns the token; *margin = distance of r to the nearest CDF edge
// of the chosen token (NaN on the degenerate one-hot path, 0 when greedy).
__device__ uint32_t sample_cta(const float* l, int V, float T, uint32_t word, float* margin, float* smem) {
  if (T == 0.0f) {
    *margin = 0.0f;
    return argmax_cta(l, V, smem);
  }
  const int nblk = (V + 255) / 256;
  const int nsb = (nblk + 31) / 32;
  float* red = smem;                // [kWarps]
  float* bsum = smem + 2 * kWarps;  // [nblk]
  __shared__ float s_total, s_Q, s_R, s_margin;
  __shared__ int s_k, s_found, s_tok;
  // max of s = l / T (NaN ignored)
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < V; i += kThreads) mx = fmaxf(mx, __fdiv_rn(ld_f(l + i), T));
  const float M = block_max(mx, red);
  // total of e
  block_sums(l, V, T, M, 0.0f, false, bsum, nblk);
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.0f;
    for (int s = 0; s < nsb; s++) {
      float sb = 0.0f;
      for (int k = s * 32; k < min(nblk, s * 32 + 32); k++) sb = __fadd_rn(sb, bsum[k]);
      tot = __fadd_rn(tot, sb);
    }
    s_total = tot;
  }
  __syncthreads();
  const float total = s_total;
  if (!(total > 0.0f) || !isfinite(total)) {
    *margin = NAN;
    return argmax_cta(l, V, smem);
  }
  const float inv = __fdiv_rn(1.0f, total);
  // block sums of p and the last index with p > 0
  block_sums(l, V, T, M, inv, true, bsum, nblk);
  int last = -1;
  for (int i = threadIdx.x; i < V; i += kThreads)
    if (prob_at(l, V, i, T, M, inv, true) > 0.0f) last = i;
  __syncthreads();
  last = block_max_int(last, reinterpret_cast<int*>(red));
  const float r = (float)(word >> 8) * (1.0f / 16777216.0f);
  if (threadIdx.x == 0) {
    float Q = 0.0f, R = 0.0f;
    int found = 0, fk = 0;
    for (int s = 0; s < nsb && !found; s++) {
      float sb = 0.0f;
      for (int k = s * 32; k < min(nblk, s * 32 + 32); k++) sb = __fadd_rn(sb, bsum[k]);
      const float Qn = __fadd_rn(Q, sb);
      if (r < Qn) {
        float Rk = 0.0f;
        fk = min(nblk, s * 32 + 32) - 1;
        for (int k = s * 32; k < min(nblk, s * 32 + 32); k++) {
          const float Rn = __fadd_rn(Rk, bsum[k]);
          if (r < __fadd_rn(Q, Rn)) {
            fk = k;
            break;
          }
          Rk = Rn;
        }
        R = Rk;
        found = 1;
        break;
      }
      Q = Qn;
    }
    s_found = found;
    s_k = fk;
    s_Q = Q;
    s_R = R;
  }
  __syncthreads();
  if (!s_found) {
    // r at or beyond the rounded CDF total: the last non-zero token
    // (sampler.rs:106-108).
    *margin = __fsub_rn(r, s_Q);
    const uint32_t result = (uint32_t)(last < 0 ? 0 : last);
    __syncthreads();
    return result;
  }
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const int i0 = s_k * 256 + lane * 8;
    float pv[8];
    float ls = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; e++) {
      pv[e] = prob_at(l, V, i0 + e, T, M, inv, true);
      ls = __fadd_rn(ls, pv[e]);
    }
    float S = 0.0f;  // sequential prefix of the lane sums before this lane
    for (int j = 0; j < 32; j++) {
      const float o = __shfl_sync(0xffffffffu, ls, j);
      if (j < lane) S = __fadd_rn(S, o);
    }
    const float Q = s_Q, R = s_R;
    const float lane_end = __fadd_rn(Q, __fadd_rn(R, __fadd_rn(S, ls)));
    const unsigned hit = __ballot_sync(0xffffffffu, r < lane_end);
    const int j = hit ? __ffs(hit) - 1 : 31;
    if (lane == j) {
      float t = 0.0f;
      float prev = __fadd_rn(Q, __fadd_rn(R, S));
      int tok = min(i0 + 7, V - 1);
      float mg = 0.0f;
      for (int e = 0; e < 8; e++) {
        t = __fadd_rn(t, pv[e]);
        const float cum = __fadd_rn(Q, __fadd_rn(R, __fadd_rn(S, t)));
        if (r < cum) {
          tok = i0 + e;
          mg = fminf(__fsub_rn(cum, r), __fsub_rn(r, prev));
          break;
        }
        prev = cum;
      }
      s_tok = tok;
      s_margin = mg;
    }
  }
  __syncthreads();
  const uint32_t result = (uint32_t)s_tok;
  *margin = s_margin;
  __syncthreads();
  return result;
}

}  // namespace defer

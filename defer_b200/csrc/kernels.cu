// Kernels of the token step: one launch per phase (the stream-ordered path)
// and the persistent token-loop kernel (all phases of many steps in one
// cooperative launch, grid barriers between phases).
#include <cuda_runtime.h>

#include <algorithm>

#include "common.h"
#include "kernels.h"
#include "phases.cuh"

namespace defer {

// ------------------------------------------------------------ grid barrier
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// All CTAs arrive on a monotonically increasing counter; every wait is
// bounded (kBarrierTimeoutNs), after which the CTA records kStTimeout in the
// status word and leaves, so a lost CTA can never hang the GPU.
constexpr unsigned long long kBarrierTimeoutNs = 2000000000ull;

__device__ __forceinline__ void grid_barrier(unsigned* bar, unsigned& target, int* status) {
  __syncthreads();
  if (threadIdx.x == 0) {
    target += gridDim.x;
    __threadfence();
    atomicAdd(bar, 1u);
    const unsigned long long t0 = globaltimer_ns();
    unsigned spins = 0;
    while ((int)(ld_acquire_u32(bar) - target) < 0) {
      if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > kBarrierTimeoutNs) {
        atomicExch(status, kStTimeout);
        break;
      }
    }
  }
  __syncthreads();
}

__device__ __forceinline__ int ld_status(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// ------------------------------------------------------ per-phase kernels
extern __shared__ float dyn_smem[];

__global__ void __launch_bounds__(kThreads) k_select(DModel m, DBatch bt, int run_step) {
  ph_select(m, bt, run_step, blockIdx.x, gridDim.x, dyn_smem);
}
__global__ void __launch_bounds__(kThreads) k_finalize(DBatch bt) { ph_finalize(bt, blockIdx.x, gridDim.x); }
template <bool BF16>
__global__ void __launch_bounds__(kThreads) k_embed(DModel m, DBatch bt) {
  ph_embed<BF16>(m, bt, blockIdx.x, gridDim.x);
}
__global__ void __launch_bounds__(kThreads) k_norm(DModel m, DBatch bt, const float* w) {
  ph_norm(m, bt, w, blockIdx.x, gridDim.x);
}
template <bool BF16, int G>
__global__ void __launch_bounds__(kThreads) k_qkv(DModel m, DBatch bt, int l) {
  ph_qkv<BF16, G>(m, bt, l, blockIdx.x, gridDim.x);
}
__global__ void __launch_bounds__(kThreads) k_attn(DModel m, DBatch bt, int l) {
  ph_attn(m, bt, l, blockIdx.x, gridDim.x, dyn_smem);
}
__global__ void __launch_bounds__(kThreads) k_combine(DModel m, DBatch bt) {
  ph_combine(m, bt, blockIdx.x, gridDim.x);
}
template <bool BF16, int G>
__global__ void __launch_bounds__(kThreads) k_oproj(DModel m, DBatch bt, int l) {
  ph_residual_gemv<BF16, G>(m, bt, m.layers[l].wo, m.QD, bt.att, m.QD, blockIdx.x, gridDim.x);
}
template <bool BF16, int G>
__global__ void __launch_bounds__(kThreads) k_gateup(DModel m, DBatch bt, int l) {
  ph_gateup<BF16, G>(m, bt, l, blockIdx.x, gridDim.x);
}
template <bool BF16, int G>
__global__ void __launch_bounds__(kThreads) k_down(DModel m, DBatch bt, int l) {
  ph_residual_gemv<BF16, G>(m, bt, m.layers[l].wdown, m.FF, bt.g, m.FF, blockIdx.x, gridDim.x);
}
template <bool BF16, int G>
__global__ void __launch_bounds__(kThreads) k_head(DModel m, DBatch bt) {
  ph_head<BF16, G>(m, bt, blockIdx.x, gridDim.x);
}

// The device sampler on an arbitrary logits vector (one CTA).
__global__ void __launch_bounds__(kThreads) k_sample_one(const float* logits, int V, float T, uint32_t word,
                                                         uint32_t* out_tok, float* out_margin) {
  float margin = 0.0f;
  uint32_t t = sample_cta(logits, V, T, word, &margin, dyn_smem);
  if (threadIdx.x == 0) {
    *out_tok = t;
    *out_margin = margin;
  }
}

void launch_sample_one(const float* logits, int V, float T, uint32_t word, uint32_t* out_tok, float* out_margin,
                       cudaStream_t st) {
  size_t smem = (size_t)(2 * kWarps + (V + 255) / 256 + 8) * sizeof(float);
  if (smem > 48 * 1024) fail(kInvalidArgument, "vocabulary too large for the sampler");
  k_sample_one<<<1, kThreads, smem, st>>>(logits, V, T, word, out_tok, out_margin);
  DEFER_CUDA(cudaGetLastError());
}

// ---------------------------------------------------- persistent kernel
// Runs up to `nsteps` token steps of every slot in the batch. Layer
// pointers are read from the device array, so the kernel argument block
// stays small.
template <bool BF16, int G>
__global__ void __launch_bounds__(kThreads, 1) k_persistent(DModel m, DBatch bt, int nsteps) {
  const int cta = blockIdx.x, ncta = gridDim.x;
  unsigned target = 0;
  for (int s = 0; s < nsteps; s++) {
    ph_select(m, bt, s, cta, ncta, dyn_smem);
    grid_barrier(bt.bar, target, bt.status);
    if (ld_status(bt.status) != kStOk) return;
    if (!ld_status(bt.any_active + (s & 1))) break;
    ph_embed<BF16>(m, bt, cta, ncta);
    grid_barrier(bt.bar, target, bt.status);
    for (int l = 0; l < m.L; l++) {
      const DLayer& Ly = m.layers[l];
      ph_norm(m, bt, Ly.attn_norm, cta, ncta);
      grid_barrier(bt.bar, target, bt.status);
      ph_qkv<BF16, G>(m, bt, l, cta, ncta);
      grid_barrier(bt.bar, target, bt.status);
      ph_attn(m, bt, l, cta, ncta, dyn_smem);
      grid_barrier(bt.bar, target, bt.status);
      ph_combine(m, bt, cta, ncta);
      grid_barrier(bt.bar, target, bt.status);
      ph_residual_gemv<BF16, G>(m, bt, Ly.wo, m.QD, bt.att, m.QD, cta, ncta);
      grid_barrier(bt.bar, target, bt.status);
      ph_norm(m, bt, Ly.ffn_norm, cta, ncta);
      grid_barrier(bt.bar, target, bt.status);
      ph_gateup<BF16, G>(m, bt, l, cta, ncta);
      grid_barrier(bt.bar, target, bt.status);
      ph_residual_gemv<BF16, G>(m, bt, Ly.wdown, m.FF, bt.g, m.FF, cta, ncta);
      grid_barrier(bt.bar, target, bt.status);
      if (ld_status(bt.status) != kStOk) return;
    }
    ph_norm(m, bt, m.norm, cta, ncta);
    grid_barrier(bt.bar, target, bt.status);
    ph_head<BF16, G>(m, bt, cta, ncta);
    grid_barrier(bt.bar, target, bt.status);
    if (ld_status(bt.status) != kStOk) return;
  }
  ph_finalize(bt, cta, ncta);
}

// ------------------------------------------------------------ launchers
static int div_up(long a, long b) { return (int)((a + b - 1) / b); }

size_t step_smem_bytes(const DModel& m) {
  const int G = m.NH / m.NKV;
  size_t attn = (size_t)(G * m.HD + G * kAttnChunk) * sizeof(float);
  size_t samp = (size_t)(2 * kWarps + (m.V + 255) / 256 + 8) * sizeof(float);
  size_t s = attn > samp ? attn : samp;
  return s < 1024 ? 1024 : s;
}

template <bool BF16, int G>
static void phased_impl(const DModel& m, const DLayer* hl, const DBatch& bt, int first_step, int nsteps, int sms,
                        cudaStream_t st) {
  const size_t smem = step_smem_bytes(m);
  const int B = bt.B;
  const int cap = sms * 8;
  auto wg = [&](long units) { return std::max(1, std::min(div_up(units, kWarps), cap)); };
  const int attn_units = B * m.NKV * bt.max_chunks;
  for (int s = 0; s < nsteps; s++) {
    k_select<<<B, kThreads, smem, st>>>(m, bt, first_step + s);
    k_embed<BF16><<<B, kThreads, 0, st>>>(m, bt);
    for (int l = 0; l < m.L; l++) {
      k_norm<<<B, kThreads, 0, st>>>(m, bt, hl[l].attn_norm);
      k_qkv<BF16, G><<<wg(m.QKVR / 2), kThreads, 0, st>>>(m, bt, l);
      k_attn<<<std::min(attn_units, cap), kThreads, smem, st>>>(m, bt, l);
      k_combine<<<std::min(B * m.NH, cap), kThreads, 0, st>>>(m, bt);
      k_oproj<BF16, G><<<wg(m.H), kThreads, 0, st>>>(m, bt, l);
      k_norm<<<B, kThreads, 0, st>>>(m, bt, hl[l].ffn_norm);
      k_gateup<BF16, G><<<wg(m.FF), kThreads, 0, st>>>(m, bt, l);
      k_down<BF16, G><<<wg(m.H), kThreads, 0, st>>>(m, bt, l);
    }
    k_norm<<<B, kThreads, 0, st>>>(m, bt, m.norm);
    k_head<BF16, G><<<wg(m.V), kThreads, 0, st>>>(m, bt);
  }
  k_finalize<<<B, kThreads, 0, st>>>(bt);
  DEFER_CUDA(cudaGetLastError());
}

static int group_for(int B) { return B <= 1 ? 1 : B <= 2 ? 2 : B <= 4 ? 4 : 8; }

void launch_steps_phased(const DModel& m, const DLayer* host_layers, const DBatch& bt, int first_step, int nsteps,
                         int sms, cudaStream_t st) {
  const int G = group_for(bt.B);
  if (m.bf16) {
    switch (G) {
      case 1: phased_impl<true, 1>(m, host_layers, bt, first_step, nsteps, sms, st); break;
      case 2: phased_impl<true, 2>(m, host_layers, bt, first_step, nsteps, sms, st); break;
      case 4: phased_impl<true, 4>(m, host_layers, bt, first_step, nsteps, sms, st); break;
      default: phased_impl<true, 8>(m, host_layers, bt, first_step, nsteps, sms, st); break;
    }
  } else {
    switch (G) {
      case 1: phased_impl<false, 1>(m, host_layers, bt, first_step, nsteps, sms, st); break;
      case 2: phased_impl<false, 2>(m, host_layers, bt, first_step, nsteps, sms, st); break;
      case 4: phased_impl<false, 4>(m, host_layers, bt, first_step, nsteps, sms, st); break;
      default: phased_impl<false, 8>(m, host_layers, bt, first_step, nsteps, sms, st); break;
    }
  }
}

template <bool BF16, int G>
static void persistent_impl(const DModel& m, const DBatch& bt, int nsteps, int sms, cudaStream_t st) {
  const size_t smem = step_smem_bytes(m);
  auto kern = k_persistent<BF16, G>;
  int per_sm = 0;
  DEFER_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem));
  if (per_sm < 1) fail(kCuda, "persistent kernel cannot be resident");
  const int grid = sms;  // one CTA per SM
  DEFER_CUDA(cudaMemsetAsync(bt.bar, 0, sizeof(unsigned), st));
  DEFER_CUDA(cudaMemsetAsync(bt.any_active, 0, 2 * sizeof(int), st));
  DModel mm = m;
  DBatch bb = bt;
  int ns = nsteps;
  void* args[] = {&mm, &bb, &ns};
  DEFER_CUDA(cudaLaunchCooperativeKernel((const void*)kern, dim3(grid), dim3(kThreads), args, smem, st));
}

void launch_steps_persistent(const DModel& m, const DBatch& bt, int nsteps, int sms, cudaStream_t st) {
  const int G = group_for(bt.B);
  if (m.bf16) {
    switch (G) {
      case 1: persistent_impl<true, 1>(m, bt, nsteps, sms, st); break;
      case 2: persistent_impl<true, 2>(m, bt, nsteps, sms, st); break;
      case 4: persistent_impl<true, 4>(m, bt, nsteps, sms, st); break;
      default: persistent_impl<true, 8>(m, bt, nsteps, sms, st); break;
    }
  } else {
    switch (G) {
      case 1: persistent_impl<false, 1>(m, bt, nsteps, sms, st); break;
      case 2: persistent_impl<false, 2>(m, bt, nsteps, sms, st); break;
      case 4: persistent_impl<false, 4>(m, bt, nsteps, sms, st); break;
      default: persistent_impl<false, 8>(m, bt, nsteps, sms, st); break;
    }
  }
}

}  // namespace defer

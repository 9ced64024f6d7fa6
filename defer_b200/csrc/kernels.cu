// Kernels of the token step: one launch per phase (the stream-ordered path)
// and the persistent token-loop kernel (all phases of many steps in one
// cooperative launch, grid barriers between phases).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>

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

__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
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

// `limit_ns` replaces the limit when non-zero; `withhold` (a fault drill set
// from the host) makes this CTA skip its arrival, so every CTA's wait runs
// out.
__device__ __forceinline__ void grid_barrier(unsigned* bar, unsigned& target, int* status,
                                             unsigned long long limit_ns = 0, bool withhold = false) {
  __syncthreads();
  if (threadIdx.x == 0) {
    target += gridDim.x;
    if (!withhold) red_release_add(bar, 1u);
    const unsigned long long lim = limit_ns ? limit_ns : kBarrierTimeoutNs;
    const unsigned long long t0 = globaltimer_ns();
    unsigned spins = 0;
    while ((int)(ld_acquire_u32(bar) - target) < 0) {
      if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > lim) {
        atomicExch(status, kStTimeout);
        break;
      }
    }
    __threadfence();
  }
  __syncthreads();
}

__device__ __forceinline__ int ld_status(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// ------------------------------------------------------ per-phase kernels
extern __shared__ __align__(16) float dyn_smem[];

template <bool BF16>
__global__ void __launch_bounds__(kThreads) k_select(DModel m, DBatch bt, int run_step) {
  ph_select<BF16>(m, bt, run_step, blockIdx.x, gridDim.x, dyn_smem);
}
__global__ void __launch_bounds__(kThreads) k_finalize(DBatch bt) { ph_finalize(bt, blockIdx.x, gridDim.x); }
template <bool BF16, int G>
__global__ void __launch_bounds__(kThreads) k_qkv(DModel m, DBatch bt, int l) {
  ph_qkv<BF16, G>(m, bt, l, blockIdx.x, gridDim.x, dyn_smem);
}
__global__ void __launch_bounds__(kThreads) k_attn(DModel m, DBatch bt, int l) {
  ph_attn_chunks(m, bt, l, blockIdx.x, gridDim.x, dyn_smem);
}
__global__ void __launch_bounds__(kThreads) k_attn_combine(DModel m, DBatch bt) {
  ph_attn_combine(m, bt, blockIdx.x, gridDim.x);
}
template <bool BF16, int G>
__global__ void __launch_bounds__(kThreads) k_oproj(DModel m, DBatch bt, int l, unsigned smem_floats) {
  ph_residual_gemv<BF16, G>(m, bt, m.layers[l].wo, m.QD, bt.att, blockIdx.x, gridDim.x, dyn_smem, smem_floats);
}
template <bool BF16, int G>
__global__ void __launch_bounds__(kThreads) k_gateup(DModel m, DBatch bt, int l) {
  ph_gateup<BF16, G>(m, bt, l, blockIdx.x, gridDim.x, dyn_smem);
}
template <bool BF16, int G>
__global__ void __launch_bounds__(kThreads) k_down(DModel m, DBatch bt, int l, unsigned smem_floats) {
  if (l + 1 < m.L)
    prefetch_rows(m.layers[l + 1].wqkv, m.QKVR, m.H, BF16, m.QKVR / 2, 2, blockIdx.x, gridDim.x);
  ph_residual_gemv<BF16, G>(m, bt, m.layers[l].wdown, m.FF, bt.g, blockIdx.x, gridDim.x, dyn_smem, smem_floats);
}
template <bool BF16, int G>
__global__ void __launch_bounds__(kThreads) k_head(DModel m, DBatch bt) {
  ph_head<BF16, G>(m, bt, blockIdx.x, gridDim.x, dyn_smem);
}
__global__ void __launch_bounds__(kThreads) k_restat(DModel m, DBatch bt) { ph_restat(m, bt, blockIdx.x, gridDim.x); }

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

size_t sample_one_smem_bytes(int V) { return sample_exact_floats(V) * sizeof(float); }

void launch_sample_one(const float* logits, int V, float T, uint32_t word, uint32_t* out_tok, float* out_margin,
                       cudaStream_t st) {
  const size_t smem = sample_one_smem_bytes(V);
  if (smem > 200 * 1024) fail(kInvalidArgument, "vocabulary too large for the one-CTA sampler");
  DEFER_CUDA(cudaFuncSetAttribute(k_sample_one, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  k_sample_one<<<1, kThreads, smem, st>>>(logits, V, T, word, out_tok, out_margin);
  DEFER_CUDA(cudaGetLastError());
}

// ---------------------------------------------------- persistent kernel
// Runs up to `nsteps` token steps of every slot in the batch. Layer
// pointers are read from the device array, so the kernel argument block
// stays small.
template <bool BF16, int G>
__global__ void __launch_bounds__(kThreads, 1) k_persistent(DModel m, DBatch bt, int nsteps, unsigned smem_floats) {
  const int cta = blockIdx.x, ncta = gridDim.x;
  unsigned target = 0;
  if (any_first(bt, false)) {  // the first step samples from the previous run's logits
    ph_restat(m, bt, cta, ncta);  // their block statistics (the greedy argmax)
    grid_barrier(bt.bar, target, bt.status, bt.wait_ns);
  }
  for (int s = 0; s < nsteps; s++) {
    ph_select<BF16>(m, bt, s, cta, ncta, dyn_smem);
    grid_barrier(bt.bar, target, bt.status, bt.wait_ns, bt.stall && s == 0 && cta == 0);
    if (ld_status(bt.status) != kStOk) return;
    if (!ld_status(bt.any_active + (s & 1))) break;
    for (int l = 0; l < m.L; l++) {
      const DLayer& Ly = m.layers[l];
      ph_qkv<BF16, G>(m, bt, l, cta, ncta, dyn_smem);
      grid_barrier(bt.bar, target, bt.status, bt.wait_ns);
      ph_attn_chunks(m, bt, l, cta, ncta, dyn_smem);
      grid_barrier(bt.bar, target, bt.status, bt.wait_ns);
      ph_attn_combine(m, bt, cta, ncta);
      grid_barrier(bt.bar, target, bt.status, bt.wait_ns);
      ph_residual_gemv<BF16, G>(m, bt, Ly.wo, m.QD, bt.att, cta, ncta, dyn_smem, smem_floats);
      grid_barrier(bt.bar, target, bt.status, bt.wait_ns);
      ph_gateup<BF16, G>(m, bt, l, cta, ncta, dyn_smem);
      grid_barrier(bt.bar, target, bt.status, bt.wait_ns);
      if (l + 1 < m.L) prefetch_rows(m.layers[l + 1].wqkv, m.QKVR, m.H, BF16, m.QKVR / 2, 2, cta, ncta);
      ph_residual_gemv<BF16, G>(m, bt, Ly.wdown, m.FF, bt.g, cta, ncta, dyn_smem, smem_floats);
      grid_barrier(bt.bar, target, bt.status, bt.wait_ns);
      if (ld_status(bt.status) != kStOk) return;
    }
    ph_head<BF16, G>(m, bt, cta, ncta, dyn_smem);
    grid_barrier(bt.bar, target, bt.status, bt.wait_ns);  // the next SELECT samples from these logits
    if (ld_status(bt.status) != kStOk) return;
  }
  ph_finalize(bt, cta, ncta);
}

// ------------------------------------------------------------ launchers
static int div_up(long a, long b) { return (int)((a + b - 1) / b); }

// Slots per register tile: enough for the batch, at most 32, and small
// enough that the group's normalised rows fit comfortably in shared memory.
static int group_for(const DModel& m, int B) {
  int G = B <= 1 ? 1 : B <= 2 ? 2 : B <= 4 ? 4 : B <= 8 ? 8 : B <= 16 ? 16 : kMaxGroupWide;
  while (G > 8 && (size_t)G * std::max(m.H, m.QD) * sizeof(float) > 96 * 1024) G /= 2;
  return G;
}

// Dynamic shared memory (floats) of the step phases for a batch of B: the
// staged activations of one slot group (normed inputs, O-projection input,
// the down-projection input when it fits), the attention chunk, and the
// sampler's group sums.
static size_t step_smem_floats(const DModel& m, int B, int max_chunks) {
  const int G = group_for(m, B);
  const int Gh = m.NH / m.NKV;
  size_t f = (size_t)G * std::max(m.H, m.QD);
  const size_t ffs = (size_t)G * m.FF;
  if (ffs * 4 <= 200 * 1024) f = std::max(f, ffs);  // the down projection's input, when it fits
  (void)max_chunks;
  // attention chunks: slot state, scores and at least two unit buffers (more
  // when the other stages leave room, up to kAttnMaxBuf)
  f = std::max(f, attn_smem_floats(B, Gh, m.HD, 1, 2));
  const size_t a2 = attn_smem_floats(B, Gh, m.HD, 2, 2);  // two CTA parts, when that fits
  if (a2 * 4 <= 200 * 1024) f = std::max(f, a2);
  // the wide head: normalized rows plus one [8][kSBlk] tile buffer per warp
  if (G >= 8) {
    f = std::max(f, (((size_t)G * m.H + 3) & ~(size_t)3) + (size_t)kPW * 8 * kSBlk);
    const size_t hs = head_staged_floats(G, m.H, m.bf16 != 0);  // staged head, when it fits
    if (hs * 4 <= 200 * 1024) f = std::max(f, hs);
  }
  // the exact sampler of SELECT
  f = std::max(f, sample_exact_floats(m.V));
  return (f + 3) & ~(size_t)3;
}

// CTA partitions of the wide projections (Part in phases.cuh). Each
// partition reads every weight of a layer through L2 once and each CTA
// re-reads the activation rows of its partition's slots, so for one layer
//   L2 bytes ~ P * W + ncta * (B / P) * X
// with W the weight bytes and X the activation bytes one slot stages; the
// minimum is at P = sqrt(ncta * B * X / W), capped by the slot groups and
// by keeping at least 8 CTAs per partition.
static int parts_for(const DModel& m, int B, int ncta) {
  const int G = group_for(m, B);
  if (G < 8) return 1;
  const int ngroups = (B + G - 1) / G;
  const double ws = m.bf16 ? 2.0 : 4.0;
  const double X = 4.0 * (2.0 * m.H + m.QD + m.FF);
  const double W = ws * ((double)m.QKVR * m.H + (double)m.H * m.QD + 3.0 * (double)m.FF * m.H);
  int P = (int)std::lround(std::sqrt((double)ncta * B * X / W));
  return std::max(1, std::min({P, ngroups, ncta / 8}));
}

size_t step_smem_bytes(const DModel& m, int B, int max_chunks) {
  return step_smem_floats(m, B, max_chunks) * sizeof(float);
}

// Always set: the default limit covers dynamic plus static shared memory,
// so a request just under 48 KB can still exceed it.
template <class K>
static void allow_smem(K kernel, size_t bytes) {
  DEFER_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
}

template <bool BF16, int G>
static void phased_impl(const DModel& m, const DLayer* hl, const DBatch& bt0, int first_step, int nsteps, int sms,
                        cudaStream_t st) {
  const size_t sf = step_smem_floats(m, bt0.B, bt0.max_chunks);
  const size_t smem = sf * sizeof(float);
  DBatch bt = bt0;
  bt.smem_bytes = (unsigned)smem;
  bt.parts = parts_for(m, bt.B, sms);
  allow_smem(k_select<BF16>, smem);
  allow_smem(k_qkv<BF16, G>, smem);
  allow_smem(k_attn, smem);
  allow_smem(k_oproj<BF16, G>, smem);
  allow_smem(k_gateup<BF16, G>, smem);
  allow_smem(k_down<BF16, G>, smem);
  allow_smem(k_head<BF16, G>, smem);
  const int B = bt.B;
  const int grid = sms;
  const int attn_units = B * m.NKV * bt.max_chunks;
  (void)hl;
  // statistics of the resident logits for slots whose first step samples
  // (the kernel skips the slots that do not)
  k_restat<<<grid, kThreads, 0, st>>>(m, bt);
  for (int s = 0; s < nsteps; s++) {
    k_select<BF16><<<B, kThreads, smem, st>>>(m, bt, first_step + s);
    for (int l = 0; l < m.L; l++) {
      k_qkv<BF16, G><<<grid, kThreads, smem, st>>>(m, bt, l);
      k_attn<<<std::min(attn_units, sms * 8), kThreads, smem, st>>>(m, bt, l);
      k_attn_combine<<<grid, kThreads, 0, st>>>(m, bt);
      k_oproj<BF16, G><<<grid, kThreads, smem, st>>>(m, bt, l, (unsigned)sf);
      k_gateup<BF16, G><<<grid, kThreads, smem, st>>>(m, bt, l);
      k_down<BF16, G><<<grid, kThreads, smem, st>>>(m, bt, l, (unsigned)sf);
    }
    k_head<BF16, G><<<grid, kThreads, smem, st>>>(m, bt);
  }
  k_finalize<<<B, kThreads, 0, st>>>(bt);
  DEFER_CUDA(cudaGetLastError());
}

int launches_per_step_phased(const DModel& m) { return 2 + 6 * m.L; }

void launch_steps_phased(const DModel& m, const DLayer* host_layers, const DBatch& bt, int first_step, int nsteps,
                         int sms, cudaStream_t st) {
  const int G = group_for(m, bt.B);
  if (m.bf16) {
    switch (G) {
      case 1: phased_impl<true, 1>(m, host_layers, bt, first_step, nsteps, sms, st); break;
      case 2: phased_impl<true, 2>(m, host_layers, bt, first_step, nsteps, sms, st); break;
      case 4: phased_impl<true, 4>(m, host_layers, bt, first_step, nsteps, sms, st); break;
      case 8: phased_impl<true, 8>(m, host_layers, bt, first_step, nsteps, sms, st); break;
      case 16: phased_impl<true, 16>(m, host_layers, bt, first_step, nsteps, sms, st); break;
      default: phased_impl<true, 32>(m, host_layers, bt, first_step, nsteps, sms, st); break;
    }
  } else {
    switch (G) {
      case 1: phased_impl<false, 1>(m, host_layers, bt, first_step, nsteps, sms, st); break;
      case 2: phased_impl<false, 2>(m, host_layers, bt, first_step, nsteps, sms, st); break;
      case 4: phased_impl<false, 4>(m, host_layers, bt, first_step, nsteps, sms, st); break;
      case 8: phased_impl<false, 8>(m, host_layers, bt, first_step, nsteps, sms, st); break;
      case 16: phased_impl<false, 16>(m, host_layers, bt, first_step, nsteps, sms, st); break;
      default: phased_impl<false, 32>(m, host_layers, bt, first_step, nsteps, sms, st); break;
    }
  }
}

template <bool BF16, int G>
static void persistent_impl(const DModel& m, const DBatch& bt, int nsteps, int sms, cudaStream_t st) {
  const size_t sf = step_smem_floats(m, bt.B, bt.max_chunks);
  auto kern = k_persistent<BF16, G>;
  // One CTA per SM: take all the shared memory the SM offers; each stage
  // copies its weight rows into what its inputs leave free.
  int dev = 0, optin = 0;
  DEFER_CUDA(cudaGetDevice(&dev));
  DEFER_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  cudaFuncAttributes fa;
  DEFER_CUDA(cudaFuncGetAttributes(&fa, kern));
  const size_t avail = (size_t)optin > fa.sharedSizeBytes + 1024 ? (size_t)optin - fa.sharedSizeBytes - 1024 : 0;
  const size_t smem = std::max(sf * sizeof(float), avail & ~(size_t)15);
  allow_smem(kern, smem);
  int per_sm = 0;
  DEFER_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem));
  if (per_sm < 1) fail(kCuda, "persistent kernel cannot be resident");
  const int grid = sms;  // one CTA per SM
  DEFER_CUDA(cudaMemsetAsync(bt.bar, 0, sizeof(unsigned), st));
  DEFER_CUDA(cudaMemsetAsync(bt.any_active, 0, 2 * sizeof(int), st));
  DModel mm = m;
  DBatch bb = bt;
  bb.smem_bytes = (unsigned)smem;
  bb.parts = parts_for(m, bb.B, grid);
  int ns = nsteps;
  unsigned sfl = (unsigned)sf;
  void* args[] = {&mm, &bb, &ns, &sfl};
  DEFER_CUDA(cudaLaunchCooperativeKernel((const void*)kern, dim3(grid), dim3(kThreads), args, smem, st));
}

template <bool BF16, int G>
static void preload_impl() {
  cudaFuncAttributes fa;
  DEFER_CUDA(cudaFuncGetAttributes(&fa, k_persistent<BF16, G>));
}

void persistent_preload(const DModel& m, int B) {
  const int G = group_for(m, B);
  if (G != 1) fail(kInvalidArgument, "persistent_preload covers single-slot batches");
  if (m.bf16) preload_impl<true, 1>();
  else preload_impl<false, 1>();
}

void launch_steps_persistent(const DModel& m, const DBatch& bt, int nsteps, int sms, cudaStream_t st) {
  const int G = group_for(m, bt.B);
  if (m.bf16) {
    switch (G) {
      case 1: persistent_impl<true, 1>(m, bt, nsteps, sms, st); break;
      case 2: persistent_impl<true, 2>(m, bt, nsteps, sms, st); break;
      case 4: persistent_impl<true, 4>(m, bt, nsteps, sms, st); break;
      case 8: persistent_impl<true, 8>(m, bt, nsteps, sms, st); break;
      case 16: persistent_impl<true, 16>(m, bt, nsteps, sms, st); break;
      default: persistent_impl<true, 32>(m, bt, nsteps, sms, st); break;
    }
  } else {
    switch (G) {
      case 1: persistent_impl<false, 1>(m, bt, nsteps, sms, st); break;
      case 2: persistent_impl<false, 2>(m, bt, nsteps, sms, st); break;
      case 4: persistent_impl<false, 4>(m, bt, nsteps, sms, st); break;
      case 8: persistent_impl<false, 8>(m, bt, nsteps, sms, st); break;
      case 16: persistent_impl<false, 16>(m, bt, nsteps, sms, st); break;
      default: persistent_impl<false, 32>(m, bt, nsteps, sms, st); break;
    }
  }
}

}  // namespace defer

// Host entry points of the token-step kernels.
#pragma once
#include <cuda_runtime.h>

#include "device.cuh"

namespace defer {

// Dynamic shared memory of the step phases for a batch of B slots.
size_t step_smem_bytes(const DModel& m, int B, int max_chunks);

// One launch per phase for `nsteps` steps (stream ordered, no grid
// barriers). `host_layers` is the host copy of m.layers.
void launch_steps_phased(const DModel& m, const DLayer* host_layers, const DBatch& bt, int first_step, int nsteps,
                         int sms, cudaStream_t st);
int launches_per_step_phased(const DModel& m);

// All phases of up to `nsteps` steps in one cooperative persistent launch
// (one CTA per SM, bounded grid barriers between phases).
void launch_steps_persistent(const DModel& m, const DBatch& bt, int nsteps, int sms, cudaStream_t st);
// Loads the device code of the persistent kernel that a batch of B slots of
// model m launches on the current device (CUDA loads modules lazily, and a
// module load allocates device memory), without launching it.
void persistent_preload(const DModel& m, int B);

// The device sampler (argmax / temperature + CDF) on one logits vector.
void launch_sample_one(const float* logits, int V, float T, uint32_t word, uint32_t* out_tok, float* out_margin,
                       cudaStream_t st);
size_t sample_one_smem_bytes(int V);

}  // namespace defer

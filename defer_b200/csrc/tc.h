// Tensor-core (tcgen05) contraction of wide batched steps that never sample
// (csrc/tc.cu): split-bf16 operands, fp32 accumulation in tensor memory.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <vector>

#include "device.cuh"

namespace defer {

constexpr int kTcM = 128;  // slots per MMA (rows of the activation operand)

// One weight matrix packed for the tensor cores (tiles of 64 rows x 64 k,
// hi and lo bf16 terms, or one term for bf16-stored weights).
struct TcMatrix {
  const unsigned char* data = nullptr;
  int N = 0, K = 0, nkb = 0, ntile = 0, wterms = 2;
};

struct TcLayer {
  const float* attn_norm = nullptr;
  const float* ffn_norm = nullptr;
  TcMatrix qkv, o, gu, down;
  int s_qkv = 1, s_o = 1, s_gu = 1, s_down = 1;  // K splits of each GEMM
};

// Activation operand and partial sums of one run.
struct TcWork {
  unsigned char* A = nullptr;
  float* Y = nullptr;
  unsigned* tickets = nullptr;  // per row tile: K splits finished (zero between GEMMs)
};

struct TcModel {
  std::vector<TcLayer> layers;
  TcMatrix head;
  int s_head = 1;
  void* arena = nullptr;  // the packed weights, then the activation operand (owned)
  float* y_buf = nullptr; // partial sums (owned)
  unsigned* tickets = nullptr;  // per row tile (owned)
  size_t bytes = 0;
  size_t max_act = 0;     // bytes of the largest activation operand
  size_t max_y = 0;       // floats of the largest partial-sum buffer
  TcWork work;
  TcModel() = default;
  TcModel(const TcModel&) = delete;
  TcModel& operator=(const TcModel&) = delete;
  ~TcModel();
};

// Packs every projection of the model (`layers`: the host copy of the
// device layer table) for the tensor cores; waits for the packing.
TcModel* tc_model_build(const DModel& m, const std::vector<DLayer>& layers, int sms, cudaStream_t st);

size_t tc_packed_bytes(int N, int K, bool bf16);
size_t tc_act_bytes(int K);
// Packs W [N][K] (fp32, or bf16 when `bf16`) into `out` (tc_packed_bytes).
TcMatrix tc_pack(const void* W, int N, int K, bool bf16, unsigned char* out, cudaStream_t st);
int tc_splits(const TcMatrix& w, int sms);
size_t tc_y_floats(const TcMatrix& w, int splits);
// bf16 terms of the activations for weights `w`: 3 when w is bf16, else 2.
int tc_aterms(const TcMatrix& w);
// A [128 slots][K] operand from x ([B][K]), RMS-normalised by nw when
// non-null, split into `aterms` bf16 terms.
void tc_prep(const float* x, const float* nw, float eps, int K, int B, const DSlotState* st, unsigned char* A,
             int aterms, cudaStream_t s, const int* active = nullptr);
// Y[slot][n] = A . W^T (the K splits' partial sums added in split order by
// the last split of each row tile; Y holds splits x [128][n_pad] floats of
// scratch). `tickets`: ntile zeroed counters, left zeroed. With `active` (a
// device flag) the launch does nothing when it is 0.
void tc_gemm(const unsigned char* A, const TcMatrix& w, float* Y, int splits, unsigned* tickets, int* status,
             cudaStream_t s, const int* active = nullptr);

// Runs nsteps token steps of a batch of at most 128 slots whose programs
// never sample, the projections on the tensor cores.
void launch_steps_tc(const DModel& m, const TcModel& tm, const DBatch& bt, int nsteps, int sms, TcWork& wk,
                     cudaStream_t st);
int launches_per_step_tc(const DModel& m);

// Y [M][N] = X [M][K] . W [N][K]^T on the tensor cores with host buffers
// (the check of the contraction itself; M <= 128).
void tc_gemm_check(int device, const float* X, int M, const float* W, int N, int K, bool w_bf16, float* Y);

}  // namespace defer

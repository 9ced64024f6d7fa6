// Allocation-free variant of the single-token forward step.
//
// Some callers cannot allocate device memory when they run a step: a
// serving process whose memory pool has already reserved the free HBM, or a
// real-time loop that must never take the driver's allocation path. For
// them the step's scratch (activations, attention partials, slot state,
// control words) lives in one file-scope device array of fixed size instead
// of buffers from cudaMalloc; the caller passes the KV cache and the logits
// buffer it owns. The array is part of this library's image, so every GPU
// that loads the library holds it until the process exits.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/defer_b200.h"
#include "common.h"
#include "kernels.h"
#include "model.h"

namespace defer {

// Largest scratch one allocation-free step may use (stated limit).
constexpr size_t kNoAllocScratchBytes = 4u << 20;  // 4 MiB

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Writes the one-step program and the zeroed slot state / control words
// into the scratch (every call starts from these values, whatever the
// previous call left there).
__global__ void k_noalloc_init(DSession s, uint32_t token, DSession* d_sess, DSlotState* d_state, uint32_t* d_tok,
                               int* ctrl, int* tickets, int n_tickets) {
  if (blockIdx.x != 0) return;
  for (int i = threadIdx.x; i < n_tickets; i += blockDim.x) tickets[i] = 0;
  if (threadIdx.x != 0) return;
  *d_tok = token;
  s.tokens = d_tok;
  *d_sess = s;
  DSlotState z;
  z.pos = s.pos;
  z.step = 0;
  z.active = 0;
  z.done = 0;
  z.was_active = 0;
  z.cur = 0;
  z.div_step = -1;
  z.div_token = 0;
  *d_state = z;
  for (int i = 0; i < 8; i++) ctrl[i] = 0;
}

namespace {
std::mutex g_addr_mu;
void* g_addr[64] = {nullptr};

// Set-up of `device` (the current device) on its first call: the device
// address of the scratch, looked up once (host code must never hand the
// array's own name to a kernel: in host code it is only a host-side
// stand-in), and the device code of this step loaded. CUDA loads modules
// lazily and a module load allocates device memory, so doing both here
// keeps every later call free of allocations.
void* scratch_address(const DModel& d, int device) {
  std::lock_guard<std::mutex> lk(g_addr_mu);
  if (device < 0 || device >= 64) fail(kInvalidArgument, "device id out of range");
  if (!g_addr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) fail(kCuda, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    cudaFuncAttributes fa;
    DEFER_CUDA(cudaFuncGetAttributes(&fa, k_noalloc_init));
    persistent_preload(d, 1);
    g_addr[device] = p;
  }
  return g_addr[device];
}

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }
}  // namespace

void forward_noalloc(Model* m, float* k_cache, float* v_cache, uint32_t cap, uint32_t pos, uint32_t token,
                     float* logits_out, cudaStream_t st) {
  const DModel& d = m->dm;
  if (!k_cache || !v_cache || !logits_out) fail(kInvalidArgument, "cache and logits buffers must not be NULL");
  if (m->tc_all)
    fail(kInvalidArgument, "this model's token loop runs on the tensor cores; the allocation-free step computes "
                           "on the CUDA cores and would not match it");
  if (cap == 0) fail(kInvalidArgument, "cache capacity must be positive");
  if (token >= (uint32_t)d.V) fail(kModel, "token id " + std::to_string(token) + " out of range");
  if (pos >= (uint32_t)d.max_seq) fail(kModel, "context length " + std::to_string(d.max_seq) + " exceeded");
  if (pos >= cap) fail(kModel, "cache capacity " + std::to_string(cap) + " exceeded");
  const int max_chunks = (int)((cap + kAttnChunk - 1) / kAttnChunk);
  // Scratch layout: control words, slot state, program, token, activations,
  // attention partials.
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  const size_t o_ctrl = take(8 * sizeof(int));
  const size_t o_state = take(sizeof(DSlotState));
  const size_t o_sess = take(sizeof(DSession));
  const size_t o_tok = take(sizeof(uint32_t));
  const int nblk = (d.V + kSBlk - 1) / kSBlk;
  const size_t o_x = take((size_t)d.H * 4);
  const size_t o_tickets = take((size_t)d.NKV * sizeof(int));
  const size_t o_stats = take((size_t)5 * nblk * 4);
  const size_t o_q = take((size_t)d.QD * 4);
  const size_t o_att = take((size_t)d.QD * 4);
  const size_t o_g = take((size_t)d.FF * 4);
  const size_t o_part = take((size_t)d.NH * max_chunks * (d.HD + 2) * 4);
  if (off > kNoAllocScratchBytes)
    fail(kInvalidArgument, "the allocation-free step needs " + std::to_string(off) +
                               " bytes of scratch for this model and cache capacity; its limit is " +
                               std::to_string(kNoAllocScratchBytes) + " bytes");

  DEFER_CUDA(cudaSetDevice(m->device));
  char* base = static_cast<char*>(scratch_address(d, m->device));
  int* ctrl = reinterpret_cast<int*>(base + o_ctrl);
  DSlotState* state = reinterpret_cast<DSlotState*>(base + o_state);
  DSession* sess = reinterpret_cast<DSession*>(base + o_sess);
  uint32_t* tok = reinterpret_cast<uint32_t*>(base + o_tok);

  DSession s;
  s.kc = k_cache;
  s.vc = v_cache;
  s.mask = nullptr;
  s.tokens = nullptr;  // set on the device to the scratch token slot
  s.words = nullptr;
  s.margins = nullptr;
  s.stop = nullptr;
  s.n_stop = 0;
  s.cap = (int)cap;
  s.pos = (int)pos;
  s.n_prompt = 1;
  s.n_total = 1;
  s.temperature = 0.0f;
  s.verify = 0;
  s.lanes = 1;
  int* tickets = reinterpret_cast<int*>(base + o_tickets);
  k_noalloc_init<<<1, 32, 0, st>>>(s, token, sess, state, tok, ctrl, tickets, d.NKV);
  DEFER_CUDA(cudaGetLastError());

  DBatch bt{};
  bt.B = 1;
  bt.sess = sess;
  bt.st = state;
  bt.x = reinterpret_cast<float*>(base + o_x);
  bt.tickets = tickets;
  bt.nblk = nblk;
  float* stats = reinterpret_cast<float*>(base + o_stats);
  bt.ss.lmax = stats;
  bt.ss.larg = reinterpret_cast<int*>(stats + nblk);
  bt.ss.smax = stats + 2 * nblk;
  bt.ss.esum = stats + 3 * nblk;
  bt.ss.psum = stats + 4 * nblk;
  bt.q = reinterpret_cast<float*>(base + o_q);
  bt.att = reinterpret_cast<float*>(base + o_att);
  bt.g = reinterpret_cast<float*>(base + o_g);
  bt.logits = logits_out;
  bt.part = reinterpret_cast<float*>(base + o_part);
  bt.max_chunks = max_chunks;
  bt.status = ctrl;
  bt.any_active = ctrl + 1;
  bt.bar = reinterpret_cast<unsigned*>(ctrl + 3);
  launch_steps_persistent(d, bt, 1, m->sms, st);
  DEFER_CUDA(cudaGetLastError());
  int status = 0;
  DEFER_CUDA(cudaMemcpyAsync(&status, ctrl, sizeof(int), cudaMemcpyDeviceToHost, st));
  DEFER_CUDA(cudaStreamSynchronize(st));
  if (status == kStTimeout) fail(kDeviceTimeout, "a grid barrier of the token step timed out");
  if (status != kStOk) fail(kModel, "the token step reported status " + std::to_string(status));
}

}  // namespace defer

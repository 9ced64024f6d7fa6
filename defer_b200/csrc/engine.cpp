#include "engine.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "common.h"
#include "flow.h"
#include "kernels.h"
#include "tc.h"

namespace defer {

bool use_persistent() {
  const char* e = getenv("DEFER_B200_PHASED");
  return !(e && e[0] == '1');
}

int loop_mode() {
  const char* e = getenv("DEFER_B200_LOOP");
  if (e && strcmp(e, "barrier") == 0) return 0;
  if (e && strcmp(e, "flow") == 0) return 2;
  return 1;
}

int replay_lanes(size_t n) {
  const char* e = getenv("DEFER_B200_REPLAY_LANES");
  long lanes = 512;
  if (e && *e) lanes = strtol(e, nullptr, 10);
  if (lanes < 1) lanes = 1;
  // short histories are cheaper one position per step (dataflow kernel)
  if (n < 64) return 1;
  return (int)std::min<long>(lanes, (long)n);
}

static uint64_t words_per_sample(float t) { return t == 0.0f ? 0 : 1; }

// Steps a lane program needs: its feeds, plus one step that only verifies
// the index after its last feed when that index is still in the program.
static int lane_steps(int n_total, int lanes, int lane) {
  if (lanes <= 1) return n_total;
  if (lane >= n_total) return 0;
  const int feeds = (n_total - lane + lanes - 1) / lanes;
  const int last = lane + (feeds - 1) * lanes;
  return feeds + (last + 1 < n_total ? 1 : 0);
}

// ------------------------------------------------------------------ Runner
Runner::Runner(const Model* m, int B, int max_cap) : m_(m), B_(B), max_cap_(max_cap) {
  if (B <= 0) fail(kInvalidArgument, "batch size must be positive");
  DEFER_CUDA(cudaSetDevice(m->device));
  const DModel& d = m->dm;
  max_chunks_ = (max_cap + kAttnChunk - 1) / kAttnChunk;
  if (max_chunks_ < 1) max_chunks_ = 1;
  nblk_ = (d.V + kSBlk - 1) / kSBlk;
  // Activation rows padded to whole 32-slot groups: a group's kernels may
  // read (never use) the rows of slots past the batch.
  const size_t Bp = ((size_t)B + kMaxGroupWide - 1) / kMaxGroupWide * kMaxGroupWide;
  DEFER_CUDA(cudaMalloc(&x_, Bp * d.H * 4));
  DEFER_CUDA(cudaMalloc(&tickets_, (size_t)B * d.NKV * sizeof(int)));
  DEFER_CUDA(cudaMalloc(&stats_, (size_t)5 * B * nblk_ * 4));
  DEFER_CUDA(cudaMalloc(&q_, Bp * d.QD * 4));
  DEFER_CUDA(cudaMalloc(&att_, Bp * d.QD * 4));
  DEFER_CUDA(cudaMalloc(&g_, Bp * d.FF * 4));
  DEFER_CUDA(cudaMalloc(&logits_, (size_t)B * d.V * 4));
  DEFER_CUDA(cudaMalloc(&part_, (size_t)B * d.NH * max_chunks_ * (d.HD + 2) * 4));
  DEFER_CUDA(cudaMalloc(&d_sess_, sizeof(DSession) * B));
  DEFER_CUDA(cudaMalloc(&d_state_, sizeof(DSlotState) * B));
  DEFER_CUDA(cudaMalloc(&d_ctrl_, 8 * sizeof(int)));
  if (B <= kMaxGroup) {
    flow_n_ = flow_tagged_words(d, B, max_chunks_, m->sms);
    DEFER_CUDA(cudaMalloc(&flow_words_, flow_n_ * sizeof(uint64_t)));
    DEFER_CUDA(cudaMemset(flow_words_, 0, flow_n_ * sizeof(uint64_t)));
  }
  DEFER_CUDA(cudaEventCreate(&ev_start_));
  DEFER_CUDA(cudaEventCreate(&ev_stop_));
}

Runner::~Runner() {
  cudaFree(x_);
  cudaFree(tickets_);
  cudaFree(stats_);
  cudaFree(q_);
  cudaFree(att_);
  cudaFree(g_);
  cudaFree(logits_);
  cudaFree(part_);
  cudaFree(d_sess_);
  cudaFree(d_state_);
  cudaFree(d_ctrl_);
  if (flow_words_) cudaFree(flow_words_);
  if (d_scratch_) cudaFree(d_scratch_);
  if (ev_start_) cudaEventDestroy(ev_start_);
  if (ev_stop_) cudaEventDestroy(ev_stop_);
}

const float* Runner::logits(int b) const { return logits_ + (size_t)b * m_->dm.V; }

void Runner::copy_logits_to(int b, Runner& dst, int db) const {
  if (dst.m_ != m_) fail(kInvalidArgument, "runners of different models");
  DEFER_CUDA(cudaMemcpyAsync(dst.logits_ + (size_t)db * m_->dm.V, logits(b), (size_t)m_->dm.V * 4,
                             cudaMemcpyDeviceToDevice, m_->stream));
}

void Runner::download_logits(int b, float* out) const {
  DEFER_CUDA(cudaMemcpy(out, logits(b), (size_t)m_->dm.V * 4, cudaMemcpyDeviceToHost));
}

void Runner::run(std::vector<SlotProgram>& progs, std::vector<SlotResult>& results) {
  const int n = (int)progs.size();
  if (n > B_) fail(kInvalidArgument, "more programs than runner slots");
  results.assign(n, SlotResult());
  if (n == 0) return;
  DEFER_CUDA(cudaSetDevice(m_->device));
  cudaStream_t st = m_->stream;
  // Pack tokens / words / stop lists / margins into one device scratch.
  std::vector<size_t> o_tok(n), o_words(n), o_stop(n), o_marg(n);
  std::vector<int> head(n);  // the program holding slot b's tokens / words / margins (its lane 0)
  size_t total = 0;
  int nsteps = 0;
  bool any_lanes = false;
  for (int b = 0; b < n; b++) {
    SlotProgram& p = progs[b];
    if (!p.cache || p.cache->model != m_) fail(kInvalidArgument, "program without a cache of this model");
    if (p.cache->cap > max_cap_) fail(kInvalidArgument, "cache larger than the runner supports");
    head[b] = b;
    if (p.lanes > 1) {
      any_lanes = true;
      if (!p.verify || p.masked || p.lane < 0 || p.lane >= p.lanes)
        fail(kInvalidArgument, "position-parallel lanes are for unmasked verified replays");
      if (p.lane > 0) {
        const SlotProgram& h = progs[b - 1];
        if (h.lanes != p.lanes || h.lane != p.lane - 1 || h.cache != p.cache)
          fail(kInvalidArgument, "lanes of one replay must be consecutive and share its cache");
        head[b] = head[b - 1];
        nsteps = std::max(nsteps, lane_steps((int)progs[head[b]].tokens.size(), p.lanes, p.lane));
        continue;  // tokens, words and margins live in the lane-0 program
      }
      if (p.n_prompt < 1) fail(kInvalidArgument, "a position-parallel replay needs a prompt");
    }
    const int ngen = (int)p.tokens.size() - p.n_prompt;
    if (ngen < 0) fail(kInvalidArgument, "n_prompt exceeds program length");
    if (p.temperature != 0.0f && (int)p.words.size() < ngen) fail(kInvalidArgument, "missing PRNG words");
    o_tok[b] = total;
    total += p.tokens.size();
    o_words[b] = total;
    total += p.temperature != 0.0f ? (size_t)ngen : 0;
    o_stop[b] = total;
    total += p.stop.size();
    o_marg[b] = total;
    total += p.want_margins ? (size_t)ngen : 0;
    nsteps = std::max(nsteps, lane_steps((int)p.tokens.size(), p.lanes, p.lane));
  }
  if (total > scratch_words_ || !d_scratch_) {
    if (d_scratch_) cudaFree(d_scratch_);
    scratch_words_ = std::max<size_t>(total, 4096);
    DEFER_CUDA(cudaMalloc(&d_scratch_, scratch_words_ * 4));
  }
  std::vector<uint32_t> hs(std::max<size_t>(total, 1));
  std::vector<DSession> sess(n);
  std::vector<DSlotState> state(n);
  for (int b = 0; b < n; b++) {
    const int h = head[b];
    SlotProgram& p = progs[h];  // the program's data (the lane-0 program of a lane group)
    const int lane = progs[b].lane, lanes = progs[b].lanes;
    const int ngen = (int)p.tokens.size() - p.n_prompt;
    if (h == b) {
      std::copy(p.tokens.begin(), p.tokens.end(), hs.begin() + o_tok[b]);
      if (p.temperature != 0.0f) std::copy(p.words.begin(), p.words.begin() + ngen, hs.begin() + o_words[b]);
      std::copy(p.stop.begin(), p.stop.end(), hs.begin() + o_stop[b]);
    }
    DSession& s = sess[b];
    s.kc = p.cache->k;
    s.vc = p.cache->v;
    s.mask = p.masked ? p.cache->mask : nullptr;
    s.tokens = d_scratch_ + o_tok[h];
    s.words = d_scratch_ + o_words[h];
    s.margins = p.want_margins ? reinterpret_cast<float*>(d_scratch_ + o_marg[h]) : nullptr;
    s.stop = d_scratch_ + o_stop[h];
    s.n_stop = (int)p.stop.size();
    s.cap = p.cache->cap;
    s.pos = (int)p.cache->len;
    s.n_prompt = p.n_prompt;
    s.n_total = (int)p.tokens.size();
    s.temperature = p.temperature;
    s.verify = p.verify ? 1 : 0;
    s.lanes = lanes;
    DSlotState& z = state[b];
    memset(&z, 0, sizeof(z));
    z.pos = (int)p.cache->len + lane;
    z.step = lane;
    z.done = lane >= (int)p.tokens.size() ? 1 : 0;
    z.div_step = -1;
  }
  DEFER_CUDA(cudaMemcpyAsync(d_scratch_, hs.data(), total * 4, cudaMemcpyHostToDevice, st));
  DEFER_CUDA(cudaMemcpyAsync(d_sess_, sess.data(), sizeof(DSession) * n, cudaMemcpyHostToDevice, st));
  DEFER_CUDA(cudaMemcpyAsync(d_state_, state.data(), sizeof(DSlotState) * n, cudaMemcpyHostToDevice, st));
  DEFER_CUDA(cudaMemsetAsync(d_ctrl_, 0, 8 * sizeof(int), st));
  DEFER_CUDA(cudaMemsetAsync(tickets_, 0, (size_t)n * m_->dm.NKV * sizeof(int), st));

  DBatch bt{};
  bt.B = n;
  bt.sess = d_sess_;
  bt.st = d_state_;
  bt.x = x_;
  bt.tickets = tickets_;
  bt.nblk = nblk_;
  {
    const size_t per = (size_t)n * nblk_;
    bt.ss.lmax = stats_;
    bt.ss.larg = reinterpret_cast<int*>(stats_ + per);
    bt.ss.smax = stats_ + 2 * per;
    bt.ss.esum = stats_ + 3 * per;
    bt.ss.psum = stats_ + 4 * per;
  }
  bt.q = q_;
  bt.att = att_;
  bt.g = g_;
  bt.logits = logits_;
  bt.part = part_;
  bt.max_chunks = max_chunks_;
  bt.status = d_ctrl_;
  bt.any_active = d_ctrl_ + 1;
  bt.bar = reinterpret_cast<unsigned*>(d_ctrl_ + 3);
  bt.smem_bytes = 0;  // set by the launchers
  bt.parts = 1;
  bt.trace = nullptr;
  bt.trace_step = -1;
  bt.stall = m_->dbg_stall;  // fault drill: one run only
  bt.wait_ns = m_->dbg_wait_ns;
  m_->dbg_stall = 0;
  m_->dbg_wait_ns = 0;
  last_steps_ = nsteps;
  const bool persistent = use_persistent();
  FlowPlan plan;
  const int mode = persistent ? loop_mode() : 0;
  // the dataflow kernel reads a step's cached rows before that step's
  // appends are known to be visible, so lanes (which read rows other lanes
  // append in the same step) take the grid-barrier kernel
  if (mode && flow_words_ && !any_lanes && !m_->tc_all) plan = flow_plan(m_->dm, n, max_chunks_, m_->sms);
  // DEFER_B200_LOOP=flow requires the dataflow kernel for the runs it can
  // take at all (position-parallel lanes and the tensor-core step are
  // other kernels by design)
  if (mode == 2 && !plan.ok && !any_lanes && !(use_tc && n <= kTcM) && !m_->tc_all)
    fail(kInvalidArgument, std::string("the dataflow token loop does not apply: ") +
                               (flow_words_ ? plan.why : "batch wider than its slot group"));
  FlowBufs fb{};
  if (plan.ok) {
    const uint64_t need = flow_tags_per_run(m_->dm, nsteps);
    if (flow_epoch_ + need >= 0xFFFFFF00ull) {
      // tags would wrap: clear every tagged word and start again
      DEFER_CUDA(cudaMemsetAsync(flow_words_, 0, flow_n_ * sizeof(uint64_t), st));
      flow_epoch_ = 1;
    }
    fb = flow_bufs(m_->dm, B_, max_chunks_, m_->sms, flow_words_);
    fb.epoch = (uint32_t)flow_epoch_;
    flow_epoch_ += need;
  }
  unsigned long long* d_trace = nullptr;
  size_t trace_words = 0;
  if (plan.ok && m_->dbg_trace_step >= 0) {
    // per-stage trace of one step (instrumentation, armed through the C ABI)
    trace_words = (size_t)plan.geo.grid * flow_stages_per_step(m_->dm) * kTraceSlots;
    DEFER_CUDA(cudaMalloc(&d_trace, trace_words * sizeof(uint64_t)));
    DEFER_CUDA(cudaMemsetAsync(d_trace, 0, trace_words * sizeof(uint64_t), st));
    bt.trace = d_trace;
    bt.trace_step = m_->dbg_trace_step;
  }
  bool tc = false;
  if (m_->tc_all) {
    // the model's arithmetic family: every run on the tensor-core step
    if (n > kTcM) fail(kInvalidArgument, "runs of this model take at most 128 slots (tensor-core step)");
    tc = true;
  } else if (use_tc && n <= kTcM && !any_lanes) {
    // DEFER_B200_TC: 0 never, 1 whenever the run qualifies, default when the
    // hidden size makes the tensor cores pay off
    const char* e = getenv("DEFER_B200_TC");
    tc = (e && e[0] == '1') || (!(e && e[0] == '0') && m_->dm.H >= 1024);
    for (int b = 0; b < n && tc; b++) tc = progs[head[b]].n_prompt == (int)progs[head[b]].tokens.size();
  }
  if (tc && !m_->tc) m_->tc = tc_model_build(m_->dm, m_->host_layers, m_->sms, st);
  DEFER_CUDA(cudaEventRecord(ev_start_, st));
  if (tc) launch_steps_tc(m_->dm, *m_->tc, bt, nsteps, m_->sms, m_->tc->work, st);
  else if (plan.ok) launch_steps_flow(m_->dm, bt, fb, plan, nsteps, st);
  else if (persistent) launch_steps_persistent(m_->dm, bt, nsteps, m_->sms, st);
  else launch_steps_phased(m_->dm, m_->host_layers.data(), bt, 0, nsteps, m_->sms, st);
  DEFER_CUDA(cudaGetLastError());
  DEFER_CUDA(cudaEventRecord(ev_stop_, st));

  int ctrl[8];
  DEFER_CUDA(cudaMemcpyAsync(state.data(), d_state_, sizeof(DSlotState) * n, cudaMemcpyDeviceToHost, st));
  DEFER_CUDA(cudaMemcpyAsync(ctrl, d_ctrl_, sizeof(ctrl), cudaMemcpyDeviceToHost, st));
  DEFER_CUDA(cudaMemcpyAsync(hs.data(), d_scratch_, total * 4, cudaMemcpyDeviceToHost, st));
  DEFER_CUDA(cudaStreamSynchronize(st));
  if (d_trace) {
    m_->dbg_trace.resize(trace_words);
    DEFER_CUDA(cudaMemcpy(m_->dbg_trace.data(), d_trace, trace_words * sizeof(uint64_t), cudaMemcpyDeviceToHost));
    DEFER_CUDA(cudaFree(d_trace));
    m_->dbg_trace_ctas = plan.geo.grid;
    m_->dbg_trace_stages = flow_stages_per_step(m_->dm);
    m_->dbg_trace_step = -1;
  }
  // Timing and algorithmic traffic of this run: weights once per step run,
  // and per token fed at position p the KV rows 0..p read and row p written.
  float ms = 0.0f;
  DEFER_CUDA(cudaEventElapsedTime(&ms, ev_start_, ev_stop_));
  const DModel& d = m_->dm;
  const double kv_row = 2.0 * d.L * d.KVD * 4.0;  // K and V of one position, all layers
  int steps_run = 0;
  double bytes = 0.0;
  uint64_t tokens = 0;
  for (int b = 0; b < n; b++) {
    const int h = head[b];
    SlotProgram& p = progs[h];
    const int ngen = (int)p.tokens.size() - p.n_prompt;
    const int lanes = progs[b].lanes, lane = progs[b].lane;
    SlotResult& r = results[b];
    r.div_step = state[b].div_step;
    r.div_token = state[b].div_token;
    int fed;  // tokens this slot fed
    if (lanes > 1) {
      fed = state[b].step > lane ? (state[b].step - lane + lanes - 1) / lanes : 0;
      fed = std::min(fed, lane < (int)p.tokens.size() ? ((int)p.tokens.size() - lane + lanes - 1) / lanes : 0);
    } else {
      fed = state[b].step;
    }
    r.steps = fed;
    if (h == b) {
      r.tokens.assign(hs.begin() + o_tok[b], hs.begin() + o_tok[b] + p.tokens.size());
      if (p.want_margins)
        r.margins.assign(reinterpret_cast<float*>(hs.data() + o_marg[b]),
                         reinterpret_cast<float*>(hs.data() + o_marg[b]) + ngen);
    }
    const double p0 = (double)sess[b].pos;
    steps_run = std::max(steps_run, fed);
    tokens += (uint64_t)fed;
    for (int j = 0; j < fed; j++) bytes += kv_row * (p0 + lane + (double)j * lanes + 2.0);
    if (lanes > 1) {
      // the lanes fed interleaved positions of one cache: its length is the
      // last position fed + 1 over every lane
      if (fed > 0) p.cache->len = std::max(p.cache->len, (size_t)(p0 + lane + (double)(fed - 1) * lanes + 1));
    } else {
      p.cache->len = (size_t)state[b].pos;
    }
  }
  bytes += (double)steps_run * (double)m_->weight_bytes;
  m_->t_device_ms += ms;
  m_->t_runs += 1;
  m_->t_launches += tc ? (uint64_t)nsteps * (uint64_t)launches_per_step_tc(d) + 2  // + restat, finalize
                       : persistent ? 1 : (uint64_t)nsteps * (uint64_t)launches_per_step_phased(d) + 1;
  m_->t_tokens += tokens;
  m_->t_bytes += bytes;
  if (ctrl[0] == kStTimeout) fail(kDeviceTimeout, "a bounded wait of the token loop timed out");
  if (ctrl[0] == kStBadToken) fail(kModel, "token id out of range");
  if (ctrl[0] == kStContext) fail(kModel, "context length " + std::to_string(m_->cfg.max_seq_len) + " exceeded");
}

// ----------------------------------------------------------------- Session
Session::Session(const Model* m, const uint8_t seed[32], float t, int cache_cap)
    : model(m), temperature(t), rng_(seed) {
  if (!(t >= 0.0f && std::isfinite(t))) fail(kModel, "temperature must be finite and >= 0");
  memcpy(base_seed, seed, 32);
  int cap = cache_cap > 0 ? cache_cap : (int)m->cfg.max_seq_len;
  cache = cache_new(m, cap);
  runner_.reset(new Runner(m, 1, cap));
}

Session::~Session() { delete cache; }

// Feeds tokens in order; stops at the first token the reference would
// reject (model.rs:417-422) and raises its error after feeding the rest.
void Session::feed_tokens(const uint32_t* t, size_t n) {
  size_t ok = 0;
  std::string err;
  for (; ok < n; ok++) {
    if (t[ok] >= model->cfg.vocab_size) {
      err = "token id " + std::to_string(t[ok]) + " out of range";
      break;
    }
    if (cache->len + ok >= model->cfg.max_seq_len) {
      err = "context length " + std::to_string(model->cfg.max_seq_len) + " exceeded";
      break;
    }
    if (cache->len + ok >= (size_t)cache->cap) {
      err = "cache capacity " + std::to_string(cache->cap) + " exceeded";
      break;
    }
  }
  if (ok) {
    std::vector<SlotProgram> progs(1);
    progs[0].cache = cache;
    progs[0].tokens.assign(t, t + ok);
    progs[0].n_prompt = (int)ok;
    std::vector<SlotResult> res;
    runner_->run(progs, res);
    history.insert(history.end(), t, t + ok);
    has_logits_ = true;
  }
  if (!err.empty()) fail(kModel, err);
}

void Session::prompt(const uint32_t* tokens, size_t n) {
  if (history.size() != prompt_len) fail(kModel, "cannot add prompt tokens after generation started");
  feed_tokens(tokens, n);
  prompt_len = history.size();
}

void Session::refeed_last() {
  uint32_t last = history.back();
  history.pop_back();
  cache->len -= 1;
  feed_tokens(&last, 1);
}

std::vector<uint32_t> Session::generate(size_t max_tokens, const std::vector<uint32_t>& stop,
                                        const std::function<int(uint32_t, uint64_t)>& on_token) {
  std::vector<uint32_t> out;
  if (max_tokens == 0) return out;
  if (!has_logits_) fail(kModel, "no context: provide a non-empty prompt");
  const size_t limit = std::min<size_t>(model->cfg.max_seq_len, cache->cap);
  const size_t room = cache->len < limit ? limit - cache->len : 0;
  const size_t n = std::min(max_tokens, room);
  const uint64_t wps = words_per_sample(temperature);
  const size_t len0 = history.size();
  const uint64_t rng0 = rng_.word_pos();
  if (n) {
    std::vector<SlotProgram> progs(1);
    SlotProgram& p = progs[0];
    p.cache = cache;
    p.tokens.assign(n, 0);
    p.n_prompt = 0;
    p.temperature = temperature;
    if (wps) {
      p.words.resize(n);
      rng_.words(rng0, n, p.words.data());
    }
    p.stop = stop;
    p.want_margins = true;
    std::vector<SlotResult> res;
    runner_->run(progs, res);
    last_margins = res[0].margins;
    const int k = res[0].steps;
    for (int i = 0; i < k; i++) {
      const uint32_t t = res[0].tokens[i];
      history.push_back(t);
      rng_.set_word_pos(rng0 + (uint64_t)(i + 1) * wps);
      out.push_back(t);
      int rc = on_token ? on_token(t, rng_.word_pos()) : 0;
      if (rc != 0) {
        // The device ran ahead: roll the cache back to this token and
        // recompute its logits (same arithmetic, same bits).
        if (i + 1 < k) {
          cache->len = len0 + i + 1;
          refeed_last();
        }
        fail((Status)rc, "token callback failed");
      }
    }
    const bool stopped = !out.empty() && std::find(stop.begin(), stop.end(), out.back()) != stop.end();
    if (stopped || (size_t)k < n) return out;
  }
  if (n < max_tokens) {
    // The next step samples (one word) and then fails to feed (model.rs:420-422).
    rng_.set_word_pos(rng_.word_pos() + wps);
    fail(kModel, "context length " + std::to_string(model->cfg.max_seq_len) + " exceeded");
  }
  return out;
}

uint32_t Session::step() {
  std::vector<uint32_t> none;
  std::vector<uint32_t> r = generate(1, none, nullptr);
  return r.at(0);
}

Checkpoint Session::checkpoint() const {
  Checkpoint c;
  memcpy(c.model_signature, model->signature, 32);
  memcpy(c.base_seed, base_seed, 32);
  c.temperature = temperature;
  c.history_tokens = history;
  c.prompt_len = (uint32_t)prompt_len;
  c.rng_word_pos = U128{rng_.word_pos(), 0};
  return c;
}

void Session::last_logits(float* out) const {
  if (!has_logits_) fail(kModel, "no logits yet");
  runner_->download_logits(0, out);
}

static void validate_checkpoint(const Model* m, const Checkpoint& ck) {
  if (memcmp(ck.model_signature, m->signature, 32) != 0)
    fail(kCheckpoint, "model signature mismatch: checkpoint " + to_hex(ck.model_signature, 32) + " vs loaded " +
                          to_hex(m->signature, 32));
  const size_t plen = ck.prompt_len;
  if (plen > ck.history_tokens.size()) fail(kCheckpoint, "prompt_len exceeds history");
  const uint64_t expected = (uint64_t)(ck.history_tokens.size() - plen) * words_per_sample(ck.temperature);
  if (ck.rng_word_pos.hi != 0 || ck.rng_word_pos.lo != expected)
    fail(kCheckpoint, "rng_word_pos " + std::to_string(ck.rng_word_pos.lo) + " inconsistent with " +
                          std::to_string(ck.history_tokens.size() - plen) + " sampled tokens (expected " +
                          std::to_string(expected) + ")");
  // Replay samples the first generated token from the prompt's logits
  // (engine.rs:104-110 fails without them).
  if (plen == 0 && !ck.history_tokens.empty()) fail(kModel, "no context: provide a non-empty prompt");
}

static SlotProgram replay_program(const Checkpoint& ck, KvCache* cache) {
  SlotProgram p;
  p.cache = cache;
  p.tokens = ck.history_tokens;
  p.n_prompt = (int)ck.prompt_len;
  p.temperature = ck.temperature;
  p.verify = true;
  const size_t ngen = ck.history_tokens.size() - ck.prompt_len;
  if (words_per_sample(ck.temperature) && ngen) {
    ChaCha8 r(ck.base_seed);
    p.words.resize(ngen);
    r.words(0, ngen, p.words.data());
  }
  return p;
}

static void free_runner(void* p) { delete static_cast<Runner*>(p); }

// The model's wide runner for position-parallel checkouts (created on first
// use, regrown when a wider or longer replay needs it).
static Runner* replay_runner_for(const Model* m, int lanes, int cap) {
  if (!m->replay_runner || m->replay_runner_B < lanes || m->replay_runner_cap < cap) {
    const int B = std::max(lanes, m->replay_runner_B);
    const int c = std::max(cap, m->replay_runner_cap);
    if (m->replay_runner) m->replay_runner_free(m->replay_runner);
    m->replay_runner = nullptr;
    m->replay_runner = new Runner(m, B, c);
    m->replay_runner_free = free_runner;
    m->replay_runner_B = B;
    m->replay_runner_cap = c;
  }
  return static_cast<Runner*>(m->replay_runner);
}

Session* Session::checkout(const Model* m, const Checkpoint& ck, int cache_cap) {
  validate_checkpoint(m, ck);
  std::unique_ptr<Session> s(new Session(m, ck.base_seed, ck.temperature, cache_cap));
  const size_t n = ck.history_tokens.size();
  for (size_t i = 0; i < n; i++)
    if (ck.history_tokens[i] >= m->cfg.vocab_size) s->feed_tokens(ck.history_tokens.data(), i + 1);  // raises
  if (n > std::min<size_t>(m->cfg.max_seq_len, s->cache->cap)) s->feed_tokens(ck.history_tokens.data(), n);  // raises
  if (n) {
    SlotProgram base = replay_program(ck, s->cache);
    base.want_margins = true;
    std::vector<SlotResult> res;
    int lanes = ck.prompt_len >= 1 ? replay_lanes(n) : 1;
    if (m->tc_all) lanes = std::min(lanes, kTcM);  // one tensor-core tile of slots
    if (lanes <= 1) {
      std::vector<SlotProgram> progs(1, std::move(base));
      s->runner_->run(progs, res);
    } else {
      Runner* wide = replay_runner_for(m, lanes, s->cache->cap);
      std::vector<SlotProgram> progs(lanes);
      for (int j = 0; j < lanes; j++) {
        SlotProgram& p = progs[j];
        if (j == 0) p = std::move(base);
        p.cache = s->cache;
        p.verify = true;
        p.lanes = lanes;
        p.lane = j;
      }
      wide->run(progs, res);
      // the first divergence in position order over the lanes
      for (int j = 1; j < lanes; j++)
        if (res[j].div_step >= 0 && (res[0].div_step < 0 || res[j].div_step < res[0].div_step)) {
          res[0].div_step = res[j].div_step;
          res[0].div_token = res[j].div_token;
        }
      // the logits of the last position become the session's
      wide->copy_logits_to((int)((n - 1) % (size_t)lanes), *s->runner_, 0);
    }
    s->last_margins = res[0].margins;
    const SlotResult& r = res[0];
    if (r.div_step >= 0)
      fail(kDivergence, "replay sampled token " + std::to_string(r.div_token) + " at position " +
                            std::to_string(r.div_step) + ", checkpoint recorded " +
                            std::to_string(ck.history_tokens[r.div_step]));
    s->history = ck.history_tokens;
    s->has_logits_ = true;
  }
  s->prompt_len = ck.prompt_len;
  s->rng_.set_word_pos((uint64_t)(n - ck.prompt_len) * words_per_sample(ck.temperature));
  return s.release();
}

// ----------------------------------------------------------- model forward
static void free_forward_runner(void* p) { delete static_cast<Runner*>(p); }

void model_forward(Model* m, KvCache* c, uint32_t token, const size_t* masked, size_t n_masked, float* logits_out) {
  if (c->model != m) fail(kInvalidArgument, "cache belongs to another model");
  if (token >= m->cfg.vocab_size) fail(kModel, "token id " + std::to_string(token) + " out of range");
  if (c->len >= m->cfg.max_seq_len) fail(kModel, "context length " + std::to_string(m->cfg.max_seq_len) + " exceeded");
  if (c->len >= (size_t)c->cap) fail(kModel, "cache capacity " + std::to_string(c->cap) + " exceeded");
  // The model owns one single-slot runner for this entry point.
  const int want = std::max<int>(c->cap, (int)m->cfg.max_seq_len);
  if (!m->fwd_runner || m->fwd_runner_cap < want) {
    if (m->fwd_runner) m->fwd_runner_free(m->fwd_runner);
    m->fwd_runner = nullptr;
    m->fwd_runner = new Runner(m, 1, want);
    m->fwd_runner_free = free_forward_runner;
    m->fwd_runner_cap = want;
  }
  Runner* fr = static_cast<Runner*>(m->fwd_runner);
  std::vector<uint32_t> bits;
  bool any = false;
  if (n_masked) {
    bits.assign((size_t)c->cap / 32 + 1, 0);
    for (size_t i = 0; i < n_masked; i++)
      if (masked[i] < c->len) {
        bits[masked[i] >> 5] |= 1u << (masked[i] & 31);
        any = true;
      }
  }
  std::vector<SlotProgram> progs(1);
  progs[0].cache = c;
  progs[0].tokens = {token};
  progs[0].n_prompt = 1;
  progs[0].masked = any;
  if (any) DEFER_CUDA(cudaMemcpy(c->mask, bits.data(), bits.size() * 4, cudaMemcpyHostToDevice));
  std::vector<SlotResult> res;
  fr->run(progs, res);
  if (any) DEFER_CUDA(cudaMemset(c->mask, 0, bits.size() * 4));
  if (logits_out) fr->download_logits(0, logits_out);
}

// ----------------------------------------------------------- batch drivers
double log_softmax_at(const float* logits, size_t n, size_t idx) {
  double mx = -INFINITY;
  for (size_t i = 0; i < n; i++)
    if ((double)logits[i] > mx) mx = (double)logits[i];
  double sum = 0.0;
  for (size_t i = 0; i < n; i++)
    if (!std::isnan(logits[i])) sum += exp((double)logits[i] - mx);
  return ((double)logits[idx] - mx) - log(sum);
}

namespace {
struct EventPair {
  cudaEvent_t a = nullptr, b = nullptr;
  EventPair() {
    DEFER_CUDA(cudaEventCreate(&a));
    DEFER_CUDA(cudaEventCreate(&b));
  }
  ~EventPair() {
    cudaEventDestroy(a);
    cudaEventDestroy(b);
  }
};
}  // namespace

void replay_batch(Model* m, const std::vector<Checkpoint>& cks, int batch, bool fingerprints,
                  std::vector<ReplayOutcome>& out, double* device_ms) {
  out.assign(cks.size(), ReplayOutcome());
  if (device_ms) *device_ms = 0.0;
  std::vector<size_t> todo;
  int cap = 1;
  for (size_t i = 0; i < cks.size(); i++) {
    try {
      validate_checkpoint(m, cks[i]);
      for (uint32_t t : cks[i].history_tokens)
        if (t >= m->cfg.vocab_size) fail(kModel, "token id " + std::to_string(t) + " out of range");
      if (cks[i].history_tokens.size() > m->cfg.max_seq_len)
        fail(kModel, "context length " + std::to_string(m->cfg.max_seq_len) + " exceeded");
      todo.push_back(i);
      cap = std::max<int>(cap, (int)cks[i].history_tokens.size());
    } catch (const Error& e) {
      out[i].status = e.status;
      out[i].message = e.what();
    }
  }
  if (todo.empty()) return;
  if (batch <= 0) batch = 1;
  batch = std::min<int>(batch, (int)todo.size());
  // Tensor-core models replay position-parallel: the 128 slots of a tile
  // are shared by the batch's sessions as lanes.
  int lanes = 1;
  if (m->tc_all) {
    batch = std::min(batch, kTcM);
    lanes = std::max(1, std::min(replay_lanes((size_t)cap), kTcM / batch));
  }
  Runner runner(m, batch * lanes, cap);
  std::vector<std::unique_ptr<KvCache>> caches;
  for (int b = 0; b < batch; b++) caches.emplace_back(cache_new(m, cap));
  EventPair ev;
  float total_ms = 0.0f;
  for (size_t w = 0; w < todo.size(); w += batch) {
    const size_t nw = std::min<size_t>(batch, todo.size() - w);
    std::vector<SlotProgram> progs;
    std::vector<int> first(nw), count(nw);  // each session's slots
    for (size_t b = 0; b < nw; b++) {
      caches[b]->len = 0;
      const Checkpoint& ck = cks[todo[w + b]];
      const int ln = (lanes > 1 && ck.prompt_len >= 1 && replay_lanes(ck.history_tokens.size()) > 1) ? lanes : 1;
      first[b] = (int)progs.size();
      count[b] = ln;
      progs.push_back(replay_program(ck, caches[b].get()));
      if (ln > 1) {
        progs.back().lanes = ln;
        for (int j = 1; j < ln; j++) {
          SlotProgram p;
          p.cache = caches[b].get();
          p.verify = true;
          p.lanes = ln;
          p.lane = j;
          progs.push_back(std::move(p));
        }
      }
    }
    std::vector<SlotResult> res;
    DEFER_CUDA(cudaEventRecord(ev.a, m->stream));
    runner.run(progs, res);
    DEFER_CUDA(cudaEventRecord(ev.b, m->stream));
    DEFER_CUDA(cudaEventSynchronize(ev.b));
    float ms = 0.0f;
    DEFER_CUDA(cudaEventElapsedTime(&ms, ev.a, ev.b));
    total_ms += ms;
    for (size_t b = 0; b < nw; b++) {
      ReplayOutcome& o = out[todo[w + b]];
      const Checkpoint& ck = cks[todo[w + b]];
      SlotResult rb = res[first[b]];
      for (int j = 1; j < count[b]; j++) {  // the first divergence in position order over the lanes
        const SlotResult& rj = res[first[b] + j];
        if (rj.div_step >= 0 && (rb.div_step < 0 || rj.div_step < rb.div_step)) {
          rb.div_step = rj.div_step;
          rb.div_token = rj.div_token;
        }
      }
      if (rb.div_step >= 0) {
        o.status = kDivergence;
        o.div_step = rb.div_step;
        o.div_token = rb.div_token;
        o.message = "replay sampled token " + std::to_string(rb.div_token) + " at position " +
                    std::to_string(rb.div_step) + ", checkpoint recorded " +
                    std::to_string(ck.history_tokens[rb.div_step]);
      } else if (fingerprints) {
        cache_fingerprint(caches[b].get(), o.fingerprint);
      }
    }
  }
  if (device_ms) *device_ms = total_ms;
}

void generate_batch(Model* m, const std::vector<GenRequest>& reqs, int batch, std::vector<std::vector<uint32_t>>& out,
                    double* device_ms) {
  out.assign(reqs.size(), {});
  if (device_ms) *device_ms = 0.0;
  int cap = 1;
  for (auto& r : reqs) {
    if (r.prompt.empty()) fail(kModel, "no context: provide a non-empty prompt");
    for (uint32_t t : r.prompt)
      if (t >= m->cfg.vocab_size) fail(kModel, "token id " + std::to_string(t) + " out of range");
    if (r.prompt.size() + r.max_tokens > m->cfg.max_seq_len)
      fail(kModel, "context length " + std::to_string(m->cfg.max_seq_len) + " exceeded");
    if (!(r.temperature >= 0.0f && std::isfinite(r.temperature))) fail(kModel, "temperature must be finite and >= 0");
    cap = std::max<int>(cap, (int)(r.prompt.size() + r.max_tokens));
  }
  if (reqs.empty()) return;
  if (batch <= 0) batch = 1;
  batch = std::min<int>(batch, (int)reqs.size());
  if (m->tc_all) batch = std::min(batch, kTcM);
  Runner runner(m, batch, cap);
  std::vector<std::unique_ptr<KvCache>> caches;
  for (int b = 0; b < batch; b++) caches.emplace_back(cache_new(m, cap));
  EventPair ev;
  float total_ms = 0.0f;
  for (size_t w = 0; w < reqs.size(); w += batch) {
    const size_t nw = std::min<size_t>(batch, reqs.size() - w);
    std::vector<SlotProgram> progs;
    for (size_t b = 0; b < nw; b++) {
      const GenRequest& r = reqs[w + b];
      caches[b]->len = 0;
      SlotProgram p;
      p.cache = caches[b].get();
      p.tokens = r.prompt;
      p.tokens.resize(r.prompt.size() + r.max_tokens, 0);
      p.n_prompt = (int)r.prompt.size();
      p.temperature = r.temperature;
      if (r.temperature != 0.0f && r.max_tokens) {
        ChaCha8 c(r.seed);
        p.words.resize(r.max_tokens);
        c.words(0, r.max_tokens, p.words.data());
      }
      progs.push_back(std::move(p));
    }
    std::vector<SlotResult> res;
    DEFER_CUDA(cudaEventRecord(ev.a, m->stream));
    runner.run(progs, res);
    DEFER_CUDA(cudaEventRecord(ev.b, m->stream));
    DEFER_CUDA(cudaEventSynchronize(ev.b));
    float ms = 0.0f;
    DEFER_CUDA(cudaEventElapsedTime(&ms, ev.a, ev.b));
    total_ms += ms;
    for (size_t b = 0; b < nw; b++) {
      const size_t np = reqs[w + b].prompt.size();
      const size_t end = std::max<size_t>(np, (size_t)res[b].steps);
      out[w + b].assign(res[b].tokens.begin() + np, res[b].tokens.begin() + end);
    }
  }
  if (device_ms) *device_ms = total_ms;
}

std::vector<uint32_t> verify_runs(const Model* m, const uint8_t seed[32], float temperature,
                                  const std::vector<uint32_t>& prompt, int runs, size_t max_tokens,
                                  const std::vector<uint32_t>& stop, uint8_t fingerprint[32]) {
  if (runs < 1) fail(kInvalidArgument, "verify needs at least one run");
  std::vector<uint32_t> ref;
  uint8_t ref_fp[32] = {0};
  for (int run = 0; run < runs; run++) {
    Session s(m, seed, temperature, 0);
    s.prompt(prompt.data(), prompt.size());
    std::vector<uint32_t> out = s.generate(max_tokens, stop, nullptr);
    uint8_t fp[32];
    cache_fingerprint(s.cache, fp);
    if (run == 0) {
      ref = out;
      memcpy(ref_fp, fp, 32);
    } else if (out != ref || memcmp(fp, ref_fp, 32) != 0) {
      fail(kDivergence, "run " + std::to_string(run) + " diverged from run 0");
    }
  }
  // Checkout must reproduce the same cache bits.
  Checkpoint ck;
  memcpy(ck.model_signature, m->signature, 32);
  memcpy(ck.base_seed, seed, 32);
  ck.temperature = temperature;
  ck.prompt_len = (uint32_t)prompt.size();
  ck.history_tokens = prompt;
  ck.history_tokens.insert(ck.history_tokens.end(), ref.begin(), ref.end());
  ck.rng_word_pos = U128{(uint64_t)ref.size() * words_per_sample(temperature), 0};
  std::unique_ptr<Session> restored(Session::checkout(m, ck, 0));
  uint8_t fp[32];
  cache_fingerprint(restored->cache, fp);
  if (memcmp(fp, ref_fp, 32) != 0) fail(kDivergence, "checkout KV cache differs from live cache");
  memcpy(fingerprint, ref_fp, 32);
  return ref;
}

void ablation_batch(Model* m, const uint32_t* context, size_t n, uint32_t target, const size_t* positions,
                    size_t n_pos, int batch, double* base_logprob, double* ablated) {
  if (n == 0) fail(kModel, "cannot ablate an empty context");
  if (target >= m->cfg.vocab_size) fail(kModel, "target token " + std::to_string(target) + " out of range");
  for (size_t i = 0; i < n_pos; i++)
    if (positions[i] + 1 >= n)
      fail(kModel, "position " + std::to_string(positions[i]) + " can not be ablated (must be < " +
                       std::to_string(n - 1) + "; the query token itself is excluded)");
  for (size_t i = 0; i < n; i++)
    if (context[i] >= m->cfg.vocab_size) fail(kModel, "token id " + std::to_string(context[i]) + " out of range");
  if (n > m->cfg.max_seq_len) fail(kModel, "context length " + std::to_string(m->cfg.max_seq_len) + " exceeded");
  const int cap = (int)n;
  std::unique_ptr<KvCache> full(cache_new(m, cap));
  std::vector<float> logits(m->cfg.vocab_size);
  {
    Runner r1(m, 1, cap);
    r1.use_tc = true;  // the variants reuse this prefix: same arithmetic as theirs
    std::vector<SlotProgram> progs(1);
    progs[0].cache = full.get();
    progs[0].tokens.assign(context, context + n);
    progs[0].n_prompt = (int)n;
    std::vector<SlotResult> res;
    r1.run(progs, res);
    r1.download_logits(0, logits.data());
    *base_logprob = log_softmax_at(logits.data(), logits.size(), target);
  }
  if (n_pos == 0) return;
  if (batch <= 0) batch = 1;
  batch = std::min<int>(batch, (int)n_pos);
  if (m->tc_all) batch = std::min(batch, kTcM);
  Runner runner(m, batch, cap);
  runner.use_tc = true;
  std::vector<std::unique_ptr<KvCache>> caches;
  for (int b = 0; b < batch; b++) caches.emplace_back(cache_new(m, cap));
  const size_t words = (size_t)cap / 32 + 1;
  for (size_t w = 0; w < n_pos; w += batch) {
    const size_t nw = std::min<size_t>(batch, n_pos - w);
    std::vector<SlotProgram> progs;
    std::vector<std::vector<uint32_t>> bits(nw);
    for (size_t b = 0; b < nw; b++) {
      const size_t p = positions[w + b];
      KvCache* c = caches[b].get();
      cache_copy_prefix(c, full.get(), p + 1, m->stream);
      c->len = p + 1;
      bits[b].assign(words, 0);
      bits[b][p >> 5] |= 1u << (p & 31);
      DEFER_CUDA(cudaMemcpyAsync(c->mask, bits[b].data(), words * 4, cudaMemcpyHostToDevice, m->stream));
      SlotProgram prog;
      prog.cache = c;
      prog.tokens.assign(context + p + 1, context + n);
      prog.n_prompt = (int)prog.tokens.size();
      prog.masked = true;
      progs.push_back(std::move(prog));
    }
    std::vector<SlotResult> res;
    runner.run(progs, res);
    for (size_t b = 0; b < nw; b++) {
      runner.download_logits((int)b, logits.data());
      ablated[w + b] = log_softmax_at(logits.data(), logits.size(), target);
      DEFER_CUDA(cudaMemset(caches[b]->mask, 0, words * 4));
    }
  }
}

}  // namespace defer

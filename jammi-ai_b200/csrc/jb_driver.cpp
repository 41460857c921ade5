// Host runtime around the encoder: memory-budget admission, the chunked
// runner with OOM batch-halving, and the multi-device embedding driver.
//
//  * jb_scheduler  -- GpuScheduler (crates/jammi-ai/src/concurrency/gpu_scheduler.rs:11-218):
//    budget = total * (1 - headroom), CAS reservation, release on drop,
//    waiters woken on release; priority accepted and ignored, as there.
//  * jb_run_chunks -- InferenceRunner::run_chunks (crates/jammi-ai/src/inference/runner.rs:176-241)
//    with is_oom_error (:243-256): on an OOM message the batch size halves
//    (floored at 1) and the same slice is retried; any other error, or OOM at
//    batch size 1, propagates.
//  * jb_generate_embeddings -- the generate_embeddings driver
//    (crates/jammi-ai/src/pipeline/embedding.rs:47-282 -> run_chunks) made
//    multi-device: rows are length-bucketed (longest first), batches are
//    pulled by one worker thread per device (one stream each, pinned
//    double-buffered staging), and embeddings land in row order in a host
//    f32 [rows, H] buffer -- the values buffer of an Arrow
//    FixedSizeList<Float32>[H] (crates/jammi-ai/src/inference/adapter/embedding.rs:32-55)
//    -- with a validity bitmap that marks empty rows null
//    (crates/jammi-ai/src/model/backend/candle.rs:785-797).
#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstring>
#include <mutex>
#include <numeric>
#include <string>
#include <thread>
#include <vector>

#include "jb_model.h"

struct jb_scheduler {
  uint64_t total = 0;
  double headroom = 0.0;
  bool unlimited = false;
  std::atomic<uint64_t> reserved{0};
  std::mutex mu;
  std::condition_variable cv;
  uint64_t usable() const {
    return static_cast<uint64_t>(static_cast<double>(total) * (1.0 - headroom));
  }
};

namespace {

jb_status err(jb_status st, const std::string& m) { return jb::record_error(st, m); }

bool is_oom_message(const char* msg) {
  if (!msg) return false;
  std::string s(msg);
  std::transform(s.begin(), s.end(), s.begin(), [](unsigned char c) { return std::tolower(c); });
  return s.find("out of memory") != std::string::npos ||
         s.find("out_of_memory") != std::string::npos ||
         s.find("outofmemory") != std::string::npos || s.find("oom") != std::string::npos;
}

bool scheduler_try(jb_scheduler* s, uint64_t bytes) {
  if (s->unlimited) return true;
  const uint64_t usable = s->usable();
  uint64_t cur = s->reserved.load(std::memory_order_acquire);
  while (true) {
    if (cur + bytes > usable || cur + bytes < cur) return false;
    if (s->reserved.compare_exchange_weak(cur, cur + bytes, std::memory_order_acq_rel,
                                          std::memory_order_acquire))
      return true;
  }
}

void scheduler_release(jb_scheduler* s, uint64_t bytes) {
  if (s->unlimited) return;
  s->reserved.fetch_sub(bytes, std::memory_order_release);
  std::lock_guard<std::mutex> lk(s->mu);
  s->cv.notify_all();
}

}  // namespace

extern "C" {

// ── scheduler ───────────────────────────────────────────────────────────────

jb_scheduler* jb_scheduler_new(uint64_t total_bytes, double headroom_fraction) {
  if (!(headroom_fraction >= 0.0 && headroom_fraction <= 1.0)) {
    err(JB_ERR_INVALID, "headroom_fraction must be between 0.0 and 1.0");
    return nullptr;
  }
  jb_scheduler* s = new jb_scheduler();
  s->total = total_bytes;
  s->headroom = headroom_fraction;
  return s;
}

jb_scheduler* jb_scheduler_new_unlimited(void) {
  jb_scheduler* s = new jb_scheduler();
  s->total = UINT64_MAX;
  s->unlimited = true;
  return s;
}

jb_scheduler* jb_scheduler_for_device(int device, double memory_fraction) {
  if (device < 0) return jb_scheduler_new_unlimited();
  size_t free_b = 0, total_b = 0;
  int prev = -1;
  cudaGetDevice(&prev);
  const bool ok = cudaSetDevice(device) == cudaSuccess &&
                  cudaMemGetInfo(&free_b, &total_b) == cudaSuccess;
  if (prev >= 0) cudaSetDevice(prev);
  if (!ok) {
    cudaGetLastError();
    return jb_scheduler_new_unlimited();  // probe failed: admission disabled
  }
  double headroom = 1.0 - memory_fraction;
  headroom = std::min(1.0, std::max(0.0, headroom));
  return jb_scheduler_new(total_b, headroom);
}

void jb_scheduler_free(jb_scheduler* s) { delete s; }

int jb_scheduler_is_unlimited(const jb_scheduler* s) { return s && s->unlimited ? 1 : 0; }

uint64_t jb_scheduler_available(const jb_scheduler* s) {
  if (!s) return 0;
  if (s->unlimited) return UINT64_MAX;
  const uint64_t u = s->usable(), r = s->reserved.load(std::memory_order_acquire);
  return r >= u ? 0 : u - r;
}

int jb_scheduler_try_acquire(jb_scheduler* s, uint64_t bytes) {
  return (s && scheduler_try(s, bytes)) ? 1 : 0;
}

jb_status jb_scheduler_acquire(jb_scheduler* s, uint64_t bytes, int priority, int64_t timeout_ms) {
  (void)priority;  // accepted and ignored, as in the reference
  if (!s) return err(JB_ERR_INVALID, "null scheduler");
  if (!s->unlimited && bytes > s->usable())
    return err(JB_ERR_OOM, "GPU memory admission: request of " + std::to_string(bytes) +
                               " bytes exceeds the budget of " + std::to_string(s->usable()) +
                               " bytes (out of memory)");
  const auto deadline = std::chrono::steady_clock::now() +
                        std::chrono::milliseconds(timeout_ms < 0 ? (int64_t(1) << 40) : timeout_ms);
  // Releases notify under the mutex, so a waiter that failed its attempt
  // while holding it cannot miss the wake-up.
  std::unique_lock<std::mutex> lk(s->mu);
  while (!scheduler_try(s, bytes)) {
    if (s->cv.wait_until(lk, deadline) == std::cv_status::timeout) {
      if (scheduler_try(s, bytes)) break;
      return err(JB_ERR_TIMEOUT, "GPU memory admission: timed out waiting for " +
                                     std::to_string(bytes) + " bytes");
    }
  }
  return err(JB_OK, "");
}

void jb_scheduler_release(jb_scheduler* s, uint64_t bytes) {
  if (s) scheduler_release(s, bytes);
}

// ── runner ──────────────────────────────────────────────────────────────────

int jb_is_oom_message(const char* msg) { return is_oom_message(msg) ? 1 : 0; }

jb_status jb_run_chunks(int64_t rows, int* batch_size, jb_forward_cb forward, void* user) {
  if (!batch_size || *batch_size < 1 || !forward || rows < 0)
    return err(JB_ERR_INVALID, "jb_run_chunks: bad argument");
  int64_t start = 0;
  char msg[1024];
  while (start < rows) {
    const int64_t len = std::min<int64_t>(*batch_size, rows - start);
    msg[0] = 0;
    const int st = forward(user, start, len, msg, sizeof(msg));
    msg[sizeof(msg) - 1] = 0;
    if (st == JB_OK) {
      start += len;
      continue;
    }
    if (is_oom_message(msg) && *batch_size > 1) {
      *batch_size = std::max(*batch_size / 2, 1);  // retry the same slice
      continue;
    }
    return err(static_cast<jb_status>(st), msg);
  }
  return err(JB_OK, "");
}

}  // extern "C"

// ── multi-device driver ─────────────────────────────────────────────────────

namespace {

struct Slot {
  jb::DriverSlot* buf = nullptr;  // the handle's persistent staging
  std::vector<int64_t> rows;      // original row index of each output row, pending scatter
};

struct Shared {
  const uint32_t* ids;
  const uint64_t* offsets;
  const std::vector<int64_t>* order;      // valid rows, longest first
  const std::vector<int64_t>* batch_off;  // batch boundaries into order
  int pooling;
  int pad_multiple;
  int H;
  float* out;
  std::atomic<int64_t> next{0};
  std::atomic<bool> abort{false};
  std::atomic<int64_t> oom_retries{0};
  std::atomic<int64_t> tokens{0};
  std::atomic<int64_t> h2d_bytes{0};
  std::atomic<int64_t> d2h_bytes{0};
  std::mutex mu;
  // per-phase seconds summed over the workers, and each worker's wall time
  double pack_s = 0, scatter_s = 0, wait_s = 0, enqueue_s = 0, setup_s = 0;
  double worker_max = 0, worker_min = 0;
  int workers_done = 0;
  void add_times(double pack, double scat, double wait, double enq, double setup, double wall) {
    std::lock_guard<std::mutex> lk(mu);
    pack_s += pack;
    scatter_s += scat;
    wait_s += wait;
    enqueue_s += enq;
    setup_s += setup;
    worker_max = workers_done ? std::max(worker_max, wall) : wall;
    worker_min = workers_done ? std::min(worker_min, wall) : wall;
    ++workers_done;
  }
  jb_status first_status = JB_OK;
  std::string first_msg;
  void fail(jb_status st, const std::string& m) {
    std::lock_guard<std::mutex> lk(mu);
    if (first_status == JB_OK) {
      first_status = st;
      first_msg = m;
    }
    abort = true;
  }
};

int64_t row_len(const Shared& sh, int64_t r) {
  return static_cast<int64_t>(sh.offsets[r + 1] - sh.offsets[r]);
}

void scatter(Shared& sh, Slot& s) {
  for (size_t i = 0; i < s.rows.size(); ++i)
    std::memcpy(sh.out + s.rows[i] * sh.H, s.buf->h_out + i * sh.H, sizeof(float) * sh.H);
  s.rows.clear();
}

using Clock = std::chrono::steady_clock;
double since(Clock::time_point t) { return std::chrono::duration<double>(Clock::now() - t).count(); }

// Sizes the handle's staging for batches of up to `rows` rows of up to
// `seq` tokens and an output width of H; reallocates only when it grows.
void ensure_stage(jb::DriverStage& st, int rows, int seq, int H) {
  const size_t ids = size_t(rows) * seq, out = size_t(rows) * H;
  if (!st.stream)
    jb::check_cuda(cudaStreamCreateWithFlags(&st.stream, cudaStreamNonBlocking), "stream");
  if (ids <= st.ids_cap && size_t(rows) <= st.rows_cap && out <= st.out_cap) return;
  jb::check_cuda(cudaStreamSynchronize(st.stream), "staging");
  const size_t ids_cap = std::max(ids, st.ids_cap), rows_cap = std::max(size_t(rows), st.rows_cap),
               out_cap = std::max(out, st.out_cap);
  for (jb::DriverSlot& s : st.slot) {
    for (void* p : {static_cast<void*>(s.h_ids), static_cast<void*>(s.h_lens), static_cast<void*>(s.h_out)})
      if (p) cudaFreeHost(p);
    for (void* p : {static_cast<void*>(s.d_ids), static_cast<void*>(s.d_lens), static_cast<void*>(s.d_out)})
      if (p) cudaFree(p);
    s.h_ids = s.h_lens = s.d_ids = s.d_lens = nullptr;
    s.h_out = s.d_out = nullptr;
  }
  st.ids_cap = st.rows_cap = st.out_cap = 0;
  for (jb::DriverSlot& s : st.slot) {
    jb::check_cuda(cudaHostAlloc(&s.h_ids, ids_cap * 4, cudaHostAllocDefault), "pinned ids");
    jb::check_cuda(cudaHostAlloc(&s.h_lens, rows_cap * 4, cudaHostAllocDefault), "pinned lens");
    jb::check_cuda(cudaHostAlloc(&s.h_out, out_cap * 4, cudaHostAllocDefault), "pinned out");
    jb::check_cuda(cudaMalloc(&s.d_ids, ids_cap * 4), "device ids");
    jb::check_cuda(cudaMalloc(&s.d_lens, rows_cap * 4), "device lens");
    jb::check_cuda(cudaMalloc(&s.d_out, out_cap * 4), "device out");
    if (!s.done) jb::check_cuda(cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming), "event");
  }
  st.ids_cap = ids_cap;
  st.rows_cap = rows_cap;
  st.out_cap = out_cap;
}

void worker(Shared& sh, jb_model* m, jb_scheduler* sched, int batch_rows, int max_seq) {
  const auto t_start = Clock::now();
  double pack_s = 0, scatter_s = 0, wait_s = 0, enqueue_s = 0, setup_s = 0;
  struct Report {  // the worker's times reach the stats on every exit path
    Shared& sh;
    const Clock::time_point& t0;
    double &pack, &scat, &wait, &enq, &setup;
    ~Report() { sh.add_times(pack, scat, wait, enq, setup, since(t0)); }
  } report{sh, t_start, pack_s, scatter_s, wait_s, enqueue_s, setup_s};
  try {
    jb::DeviceGuard g(m->device);
    std::lock_guard<std::mutex> job(m->drv_mu);  // one job at a time on a handle's staging
    jb::DriverStage& stage = m->drv;
    auto t = Clock::now();
    ensure_stage(stage, batch_rows, max_seq, sh.H);
    setup_s += since(t);
    cudaStream_t stream = stage.stream;
    Slot slots[2];
    for (int i = 0; i < 2; ++i) slots[i].buf = &stage.slot[i];
    // a failed job leaves no copy in flight on the staging it hands back
    struct Drain {
      cudaStream_t s;
      ~Drain() { cudaStreamSynchronize(s); }
    } drain{stream};
    {
      int bs = batch_rows;  // halves on OOM, like run_chunks
      // Admission: the handle's workspace for (bs, max_seq) must fit this
      // device's budget; halve until it does, then hold the reservation for
      // the worker's lifetime (the reference holds a model's permit for the
      // lifetime of its cache entry, crates/jammi-ai/src/model/cache.rs:27-33).
      uint64_t reserved = 0;
      if (sched) {
        while (bs > 1 && jb_estimate_batch_bytes(m, bs, max_seq) > jb_scheduler_available(sched)) {
          bs = std::max(bs / 2, 1);
          sh.oom_retries++;
        }
        reserved = jb_estimate_batch_bytes(m, bs, max_seq);
        const jb_status st = jb_scheduler_acquire(sched, reserved, 0, 600000);
        if (st != JB_OK) jb::fail(st, jb_last_error());
      }
      struct Release {
        jb_scheduler* s;
        uint64_t b;
        ~Release() {
          if (s && b) jb_scheduler_release(s, b);
        }
      } release_on_exit{sched, reserved};
      int k = 0;
      const auto& order = *sh.order;
      const auto& boff = *sh.batch_off;
      const int64_t nb = static_cast<int64_t>(boff.size()) - 1;
      while (!sh.abort) {
        const int64_t b = sh.next.fetch_add(1);
        if (b >= nb) break;
        int64_t i = boff[b];
        const int64_t end = boff[b + 1];
        while (i < end && !sh.abort) {
          const int64_t len = std::min<int64_t>(bs, end - i);
          Slot& s = slots[k & 1];
          jb::DriverSlot& sb = *s.buf;
          t = Clock::now();
          jb::check_cuda(cudaEventSynchronize(sb.done), "slot wait");
          wait_s += since(t);
          t = Clock::now();
          scatter(sh, s);
          scatter_s += since(t);
          t = Clock::now();
          // pad width: the longest row of the sub-batch (rows are sorted longest first)
          int S = static_cast<int>(row_len(sh, order[i]));
          for (int64_t j = i; j < i + len; ++j) S = std::max<int>(S, static_cast<int>(row_len(sh, order[j])));
          if (sh.pad_multiple > 1) S = ((S + sh.pad_multiple - 1) / sh.pad_multiple) * sh.pad_multiple;
          S = std::min(S, max_seq);
          int64_t toks = 0;
          for (int64_t j = 0; j < len; ++j) {
            const int64_t r = order[i + j];
            const int64_t n = row_len(sh, r);
            std::memcpy(sb.h_ids + j * S, sh.ids + sh.offsets[r], n * 4);
            if (n < S) std::memset(sb.h_ids + j * S + n, 0, (S - n) * 4);
            sb.h_lens[j] = static_cast<uint32_t>(n);
            toks += n;
          }
          pack_s += since(t);
          t = Clock::now();
          jb::check_cuda(cudaMemcpyAsync(sb.d_ids, sb.h_ids, size_t(len) * S * 4, cudaMemcpyHostToDevice, stream), "H2D");
          jb::check_cuda(cudaMemcpyAsync(sb.d_lens, sb.h_lens, size_t(len) * 4, cudaMemcpyHostToDevice, stream), "H2D");
          const jb_status st = jb_encode_text_device(m, sb.d_ids, sb.d_lens, static_cast<int>(len), S,
                                                     sh.pooling, sb.d_out, stream);
          enqueue_s += since(t);
          if (st != JB_OK) {
            const std::string msg = jb_last_error();
            if (is_oom_message(msg.c_str()) && bs > 1) {
              bs = std::max(bs / 2, 1);
              sh.oom_retries++;
              continue;  // retry the same rows at half the batch size
            }
            jb::fail(st, msg);
          }
          jb::check_cuda(cudaMemcpyAsync(sb.h_out, sb.d_out, size_t(len) * sh.H * 4, cudaMemcpyDeviceToHost, stream), "D2H");
          jb::check_cuda(cudaEventRecord(sb.done, stream), "event");
          s.rows.assign(order.begin() + i, order.begin() + i + len);
          sh.tokens += toks;
          sh.h2d_bytes += static_cast<int64_t>(len) * (S + 1) * 4;
          sh.d2h_bytes += static_cast<int64_t>(len) * sh.H * 4;
          i += len;
          ++k;
        }
      }
      for (Slot& s : slots) {
        t = Clock::now();
        jb::check_cuda(cudaEventSynchronize(s.buf->done), "drain");
        wait_s += since(t);
        t = Clock::now();
        scatter(sh, s);
        scatter_s += since(t);
      }
      jb::check_device_flag(m, stream);
    }
  } catch (const jb::Error& e) {
    sh.fail(e.status, e.msg);
  } catch (const std::exception& e) {
    sh.fail(JB_ERR_INVALID, e.what());
  }
}

}  // namespace

extern "C" jb_status jb_generate_embeddings(jb_model** models, int n_models, const uint32_t* ids,
                                            const uint64_t* offsets, int64_t rows,
                                            const jb_generate_opts* opts, float* out,
                                            uint8_t* validity, jb_generate_stats* stats) {
  try {
    if (!models || n_models < 1 || !offsets || rows < 0 || !opts || !out || (rows > 0 && !ids))
      return err(JB_ERR_INVALID, "jb_generate_embeddings: bad argument");
    if (opts->batch_rows < 1) return err(JB_ERR_INVALID, "batch_rows must be >= 1");
    // text encoders: the BERT family, or the OpenCLIP text tower (its rows end
    // at their EOT token, the zero padding after it is never reached)
    const int family = models[0] ? models[0]->family : -1;
    if (family != JB_FAMILY_BERT && family != JB_FAMILY_CLIP_TEXT)
      return err(JB_ERR_INVALID, "all models must be text encoders of the same width");
    const int H = jb::output_dim(models[0]);
    int max_seq = 1 << 30;
    for (int i = 0; i < n_models; ++i) {
      if (!models[i] || models[i]->family != family || jb::output_dim(models[i]) != H)
        return err(JB_ERR_INVALID, "all models must be text encoders of the same width");
      for (int j = 0; j < i; ++j)
        if (models[j]->device == models[i]->device)
          return err(JB_ERR_INVALID, "one model handle per device");
      max_seq = std::min(max_seq, models[i]->max_pos);
    }
    const auto t0 = std::chrono::steady_clock::now();
    int64_t longest = 0, valid = 0;
    for (int64_t r = 0; r < rows; ++r) {
      if (offsets[r + 1] < offsets[r]) return err(JB_ERR_INVALID, "offsets must be non-decreasing");
      const int64_t n = static_cast<int64_t>(offsets[r + 1] - offsets[r]);
      longest = std::max(longest, n);
      valid += n > 0;
    }
    if (longest > max_seq)
      return err(JB_ERR_SEQ_TOO_LONG, "a row of " + std::to_string(longest) +
                                          " tokens exceeds max_position_embeddings " +
                                          std::to_string(max_seq));
    // Valid rows, longest first when bucketing: a counting sort over the
    // lengths (<= max_seq), stable, so equal lengths keep row order.  Empty
    // rows are left out: they are the zero vector + null (candle.rs:785-797),
    // and only their output rows are cleared here -- every other row is
    // written by the workers.
    std::vector<int64_t> order(static_cast<size_t>(valid));
    if (opts->sort_by_length) {
      std::vector<int64_t> start(static_cast<size_t>(longest) + 2, 0);
      for (int64_t r = 0; r < rows; ++r) {
        const int64_t n = static_cast<int64_t>(offsets[r + 1] - offsets[r]);
        if (n > 0) ++start[static_cast<size_t>(longest - n + 1)];
      }
      for (size_t i = 1; i < start.size(); ++i) start[i] += start[i - 1];
      for (int64_t r = 0; r < rows; ++r) {
        const int64_t n = static_cast<int64_t>(offsets[r + 1] - offsets[r]);
        if (n > 0) order[static_cast<size_t>(start[static_cast<size_t>(longest - n)]++)] = r;
      }
    } else {
      size_t i = 0;
      for (int64_t r = 0; r < rows; ++r)
        if (offsets[r + 1] > offsets[r]) order[i++] = r;
    }
    for (int64_t r = 0; r < rows; ++r)
      if (offsets[r + 1] == offsets[r]) std::memset(out + r * H, 0, sizeof(float) * H);
    std::vector<int64_t> boff;
    for (int64_t i = 0; i < static_cast<int64_t>(order.size()); i += opts->batch_rows) boff.push_back(i);
    boff.push_back(static_cast<int64_t>(order.size()));
    const double prepare_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    Shared sh;
    sh.ids = ids;
    sh.offsets = offsets;
    sh.order = &order;
    sh.batch_off = &boff;
    sh.pooling = opts->pooling;
    sh.pad_multiple = std::max(1, opts->pad_multiple);
    sh.H = H;
    sh.out = out;
    std::vector<jb_scheduler*> scheds(n_models, nullptr);
    if (opts->memory_fraction > 0)
      for (int i = 0; i < n_models; ++i)
        scheds[i] = jb_scheduler_for_device(models[i]->device, opts->memory_fraction);
    const int seq_cap = static_cast<int>(std::min<int64_t>(longest < 1 ? 1 : longest, max_seq) +
                                         sh.pad_multiple);
    std::vector<std::thread> threads;
    for (int i = 0; i < n_models; ++i)
      threads.emplace_back(worker, std::ref(sh), models[i], scheds[i], opts->batch_rows,
                           std::min(seq_cap, max_seq));
    for (auto& t : threads) t.join();
    for (jb_scheduler* s : scheds) jb_scheduler_free(s);
    if (sh.first_status != JB_OK) return err(sh.first_status, sh.first_msg);
    if (validity) {
      std::memset(validity, 0, static_cast<size_t>((rows + 7) / 8));
      for (int64_t r : order) validity[r >> 3] |= static_cast<uint8_t>(1u << (r & 7));
    }
    if (stats) {
      stats->rows = rows;
      stats->valid_rows = static_cast<int64_t>(order.size());
      stats->batches = static_cast<int64_t>(boff.size()) - 1;
      stats->tokens = sh.tokens;
      stats->oom_retries = sh.oom_retries;
      stats->seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
      stats->h2d_bytes = sh.h2d_bytes;
      stats->d2h_bytes = sh.d2h_bytes;
      stats->prepare_seconds = prepare_s;
      stats->pack_seconds = sh.pack_s;
      stats->scatter_seconds = sh.scatter_s;
      stats->wait_seconds = sh.wait_s;
      stats->enqueue_seconds = sh.enqueue_s;
      stats->setup_seconds = sh.setup_s;
      stats->worker_seconds_max = sh.worker_max;
      stats->worker_seconds_min = sh.worker_min;
    }
    return err(JB_OK, "");
  } catch (const jb::Error& e) {
    return err(e.status, e.msg);
  } catch (const std::exception& e) {
    return err(JB_ERR_INVALID, e.what());
  }
}

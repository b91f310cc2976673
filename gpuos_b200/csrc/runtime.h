// Host runtime of the aggregated small-op executor (C++, no torch).
//
// One Executor per GPU.  It turns tensor views into 128-byte request records,
// gathers them into batches, detects read/write hazards between the requests
// of a batch (and between in-flight batches), and publishes the batches either
// to the persistent worker (doorbell in mapped pinned memory) or as one
// stream-ordered kernel launch each.
//
// Reference correspondence (pytorch_ext/gpuos_ext.cpp):
//   Executor::submit_ew       build_binary_task/build_unary_task + submit_* (:137-201, :459-493, :695-707)
//   Executor::submit_reduce   build_reduce_task + submit_reduce (:827-856)
//   Executor::flush           flush (:496-622) with enqueue_task_host_to_device (:297-319)
//   Executor::register_*      ensure_elementwise_registered / ensure_reduce_registered (:681-692, :814-825)
//   Executor::ensure_worker   ensure_worker_alive (:111-126)
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/gpuos_b200.h"
#include "gpuos_abi.h"
#include "jit.h"

namespace gpuos {

struct GError : std::runtime_error {
  int code;
  GError(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

// Byte (or element) extent [lo, hi) touched by a tensor view.
struct Extent {
  uint64_t lo = 0, hi = 0;
  bool empty() const { return hi <= lo; }
};

// Disjoint union of extents: a sorted flat vector of [lo, hi) with touching
// extents merged.  Extents below or above everything held (the usual case for
// slab-allocated tensors, which arrive in address order) are answered and
// appended in O(1); others take a binary search.  clear() keeps the capacity,
// so a warmed-up set does not allocate.
class IntervalSet {
 public:
  bool overlaps(const Extent& e) const;
  void add(Extent e);
  void clear() { v_.clear(); }
  bool empty() const { return v_.empty(); }
  // the smallest extent covering the set (empty when the set is)
  Extent hull() const { return v_.empty() ? Extent{} : Extent{v_.front().lo, v_.back().hi}; }
  size_t size() const { return v_.size(); }

 private:
  std::vector<Extent> v_;
};

// FIFO ring allocator: allocations are freed in allocation order.
class RingAlloc {
 public:
  void init(uint64_t cap) { cap_ = cap; live_.clear(); }
  // returns false when the ring has no room right now
  bool alloc(uint64_t size, uint64_t tag, uint64_t* off);
  // free allocations from the front whose tag < upto
  void free_before(uint64_t upto);
  // give back the most recent allocation
  void undo_last() { if (!live_.empty()) live_.pop_back(); }
  uint64_t cap() const { return cap_; }
  bool empty() const { return live_.empty(); }

 private:
  struct Blk { uint64_t off, size, tag; };
  uint64_t cap_ = 0;
  std::deque<Blk> live_;
};

// A request waiting for the next flush.
struct Pending {
  // No zero fill of the record or the extension record: build_ew /
  // build_reduce write the whole record, and the extension record is read
  // only when has_ext.  (Value-initialising the ~600 bytes showed up in the
  // per-request submit cost.)
  Pending() {}
  Req r;
  bool has_ext = false;
  ExtRec ext;
  Extent out_ext;
  Extent in_ext[4];
  int nin = 0;
  uint32_t nchunk = 0;
  uint64_t partials = 0;  // floats of scratch this request needs
  uint64_t counters = 0;  // combine counters this request needs
};

struct InFlight {
  uint64_t seq;
  uint64_t nreq;
};

class Executor {
 public:
  Executor(int device, const gpuos_options& opt);
  ~Executor();

  // submission (thread-safe)
  void submit_ew(int op, bool is_slot, float p0, float p1, const gpuos_tensor* a,
                 const gpuos_tensor* b, const gpuos_tensor& out);
  void submit_nary(int slot, const gpuos_tensor* const* ins, int nin, const gpuos_tensor& out);
  void submit_reduce(int op, bool is_slot, const gpuos_tensor& x, const gpuos_tensor& out,
                     const int32_t* axes, int naxes, bool keepdim);
  void submit_task(const void* task);

  uint64_t flush(bool sync, cudaStream_t stream);
  void wait(uint64_t ticket, double timeout_s);
  bool poll(uint64_t ticket);  // every batch before `ticket` done (raises a batch's error)

  // jump table
  int register_elementwise(const std::string& key, const std::string& expr, int arity);
  int register_reduce(const std::string& key, const std::string& op_name);
  void set_alias(int logical, int physical);
  void set_slot(int slot, int variant, float p0, float p1);
  void get_slot(int slot, int* variant, float* p0, float* p1, int* alias);

  // per-launch CUDA-event timing of the batch kernel (stream mode)
  void set_timing(bool on);
  size_t take_timings(float* ms, size_t cap);

  // worker control
  void set_yield_every(uint64_t every);
  void set_debug_level(int level);
  void stall_next_batch();
  bool worker_alive();
  void stats(gpuos_stats* out);
  void shutdown();

  int device() const { return device_; }

 private:
  void publish(std::unique_lock<std::mutex>& lk, std::vector<Pending>& reqs, size_t i, size_t j,
               cudaStream_t stream);
  bool lean_eligible(const Pending& p, int v) const;
  bool publish_lean(std::unique_lock<std::mutex>& lk, std::vector<Pending>& reqs, size_t i,
                    uint32_t n, const std::vector<int>& var, const std::vector<uint32_t>& order,
                    uint64_t nchunk, cudaStream_t stream);
  uint32_t take_batch_err(uint64_t seq);
  void raise_batch_error_locked(uint64_t ticket);
  void reclaim();
  void ensure_worker_locked();
  void launch_worker_locked(uint64_t start);
  void ensure_scratch_locked();
  bool wait_for_room_locked(std::unique_lock<std::mutex>& lk, uint64_t bytes, uint64_t floats,
                            uint64_t counters, uint64_t* arena_off, uint64_t* part_off,
                            uint64_t* cnt_off, uint64_t seq);

  int device_;
  gpuos_options opt_;
  int sm_count_ = 0;
  int block_ = 512;
  int grid_ = 0;                // persistent worker grid (ingest CTA included)
  int batch_bps_ = 1;           // stream kernel: resident blocks per SM
  int ew_bps_ = 1, red_bps_ = 1;  // the same for the elementwise-only / reduction-only kernels
  int total_warps_ = 1;         // warps that execute a batch (chunk sizing)
  uint64_t idle_ns_ = 0, wait_limit_ns_ = 0;
  double sync_timeout_s_ = 60.0;

  cudaStream_t s_worker_ = nullptr, s_ctrl_ = nullptr, s_own_ = nullptr;
  // stream mode: payload copies run here, ahead of the launch stream
  cudaStream_t s_copy_ = nullptr;

  // mapped pinned host memory
  uint8_t* arena_ = nullptr;
  uint8_t* arena_dev_ = nullptr;
  uint64_t arena_bytes_ = 0;
  uint8_t* hostblk_ = nullptr;  // HostCtrl + Pub ring + done ring + retired ring
  HostCtrl* hctrl_ = nullptr;
  Pub* pub_ = nullptr;
  volatile uint64_t* done_ring_ = nullptr;
  volatile uint64_t* retired_ring_ = nullptr;
  volatile uint64_t* dur_ring_ = nullptr;  // device ns of each completed batch (worker, lean)
  uint8_t* stop_src_ = nullptr;            // a UINT64_MAX word: source of the stop_at reset
  uint8_t* hostblk_dev_ = nullptr;

  // device memory
  uint8_t* ring_ = nullptr;
  BatchState* states_ = nullptr;   // device: per-batch counters, kDoneRing slots
  DevCtrl* dctrl_ = nullptr;
  float* partials_ = nullptr;
  uint64_t partials_cap_ = 0;
  uint32_t* counters_ = nullptr;
  uint64_t counters_cap_ = 0;

  RingAlloc arena_alloc_, part_alloc_, cnt_alloc_;

  std::mutex mu_;
  std::vector<Pending> pending_;
  uint64_t next_seq_ = 0;
  uint64_t done_wm_ = 0;     // batches < done_wm_ are done
  uint64_t retired_wm_ = 0;  // batches < retired_wm_ are retired
  uint64_t err_seq_ = UINT64_MAX;
  uint32_t err_bits_ = 0;
  IntervalSet live_out_, live_in_;
  cudaStream_t last_stream_ = nullptr;
  bool have_last_stream_ = false;
  cudaEvent_t last_event_ = nullptr;
  bool timing_ = false;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> timed_;
  std::vector<cudaEvent_t> ev_pool_;
  std::vector<cudaEvent_t> done_ev_ = std::vector<cudaEvent_t>(kDoneRing, nullptr);  // stream mode
  std::vector<cudaEvent_t> copy_ev_ = std::vector<cudaEvent_t>(kDoneRing, nullptr);  // stream mode
  std::string cuda_err_;        // first CUDA error a completion query reported

  Tables tab_;
  Tables* dtab_ = nullptr;   // device copy, read by the persistent worker (slot requests)
  void push_tables_locked();
  std::unordered_map<std::string, int> slot_of_key_;
  // custom expressions (variants V_JIT_BASE + k) and the batch kernel linked with them
  std::vector<std::string> jit_exprs_;
  std::vector<JitKernel> jit_kernels_;  // every one linked so far (in-flight batches may use any)
  BatchState* jit_state_ = nullptr;     // persistent mode: counters of custom-expression batches
  volatile uint64_t* jit_word_ = nullptr;  // persistent mode: their error word (mapped)
  int variant_of(const Pending& p) const;
  void run_jit_batch_sync_locked(std::unique_lock<std::mutex>& lk, uint64_t aoff, uint64_t bytes,
                                 uint64_t ngran, BatchHdr* h);
  int next_slot_ = 20;       // slots below 20 are reserved as in the reference (gpuos_ext.cpp:95)

  bool started_ = false;
  bool worker_launched_ = false;
  uint64_t relaunches_ = 0;
  uint64_t requests_ = 0;
  uint64_t errors_ = 0;
  uint64_t dev_ns_ = 0;
  uint64_t lean_count_ = 0;
  int debug_level_ = 0;
  bool stall_next_ = false;  // fault injection: next staged batch waits for a chunk that never comes

  // lean batches (stream mode): whole batch in the kernel's parameters, launched
  // with programmatic dependent launch, completed by a word in done_ring_
  bool lean_on_ = true;
  bool chain_on_ = true;      // small staged batches on one cluster (GPUOS_CHAIN=0: off)
  uint64_t chain_count_ = 0;  // batches run that way
  int lean_grid_ = 0;                 // CTAs of the lean kernel (one per SM)
  int lean_warps_ = 0;                // warps of a full lean grid
  std::vector<uint8_t> lean_seq_ = std::vector<uint8_t>(kDoneRing, 0);  // batch seq is lean
  std::vector<uint8_t> lean_buf_;     // parameter block being built (largest size class)
  bool lean_prev_in_flush_ = false;   // the last op this flush put on the stream is a lean batch
  IntervalSet lean_out_, lean_in_;    // extents of this flush's lean batches
};

// Request planning (no GPU needed): broadcasting, dim coalescing, layout
// choice, vector-path legality and chunking of one request.
void build_ew(Pending& p, int op, bool is_slot, float p0, float p1, const gpuos_tensor* a,
              const gpuos_tensor* b, const gpuos_tensor& out);
void build_ew_nary(Pending& p, int op, bool is_slot, float p0, float p1,
                   const gpuos_tensor* const* ins, int nin, const gpuos_tensor& out);
void build_reduce(Pending& p, int op, bool is_slot, const gpuos_tensor& x,
                  const gpuos_tensor& out, const int32_t* axes, int naxes, bool keepdim);

// helpers shared with the tests of the host logic
uint32_t fdiv_magic(uint32_t d, uint32_t* shift);
int chunk_weight(int variant);
int variant_by_name(const std::string& name);
// Match an fp32 expression against the reference scheduler's expression
// table; returns the variant (and parameters) or -1.
int match_builtin_expr(const std::string& expr, int arity, float* p0, float* p1);

}  // namespace gpuos

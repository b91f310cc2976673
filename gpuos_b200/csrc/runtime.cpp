// Host runtime of the aggregated small-op executor and its C ABI.
// See runtime.h for the structure and the reference correspondence.
#include "runtime.h"

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstddef>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <thread>

#if defined(__x86_64__)
#include <immintrin.h>
#define GPUOS_PAUSE() _mm_pause()
#else
#define GPUOS_PAUSE() std::this_thread::yield()
#endif

extern "C" cudaError_t gpuos_launch_batch(const uint8_t* payload, const gpuos::BatchHdr* hdr,
                                          gpuos::BatchState* st, volatile uint64_t* done_ring,
                                          uint64_t wait_limit_ns, int grid, cudaStream_t stream,
                                          int bodies);
extern "C" cudaError_t gpuos_launch_worker(const void* args, int grid, cudaStream_t stream);
extern "C" cudaError_t gpuos_launch_chain(const uint8_t* payload, const gpuos::BatchHdr* hdr,
                                          gpuos::BatchState* st, volatile uint64_t* done_ring,
                                          uint64_t wait_limit_ns, int ctas, cudaStream_t stream);
extern "C" cudaError_t gpuos_occupancy(int* batch_blocks_per_sm, int* worker_blocks_per_sm,
                                       int* ew_blocks_per_sm, int* red_blocks_per_sm);
extern "C" int gpuos_cta_threads();
extern "C" cudaError_t gpuos_launch_lean(const void* params, int size_class, int grid,
                                         cudaStream_t stream);
extern "C" size_t gpuos_lean_params_size(int size_class);

namespace gpuos {

namespace {

thread_local std::string t_last_error;

#define GCU(expr)                                                                     \
  do {                                                                                \
    cudaError_t e_ = (expr);                                                          \
    if (e_ != cudaSuccess)                                                            \
      throw GError(GPUOS_ECUDA, std::string(#expr) + ": " + cudaGetErrorString(e_));  \
  } while (0)

constexpr uint64_t kDoneMask = (1ull << 48) - 1;

inline bool dt_ok(int dt) { return dt == kF32 || dt == kF16 || dt == kBF16; }
inline int esz(int dt) { return dt == kF32 ? 4 : 2; }
inline uint64_t align_up(uint64_t x, uint64_t a) { return (x + a - 1) / a * a; }
inline uint32_t pow2_ceil(uint64_t x) {
  uint32_t p = 1;
  while (p < x && p < (1u << 30)) p <<= 1;
  return p;
}

void check_tensor(const gpuos_tensor& t, const char* what) {
  if (t.ndim < 0 || t.ndim > kMaxDims)
    throw GError(GPUOS_EINVAL, std::string(what) + ": ndim must be in [0, 8]");
  if (!dt_ok(t.dtype))
    throw GError(GPUOS_EINVAL, std::string(what) +
                                   ": dtype must be float32, float16 or bfloat16 (code " +
                                   std::to_string(t.dtype) + ")");
  for (int d = 0; d < t.ndim; ++d)
    if (t.sizes[d] < 0) throw GError(GPUOS_EINVAL, std::string(what) + ": negative size");
}

int64_t numel_of(const gpuos_tensor& t) {
  int64_t n = 1;
  for (int d = 0; d < t.ndim; ++d) n *= t.sizes[d];
  return n;
}

Extent extent_of(const gpuos_tensor& t) {
  int64_t lo = 0, hi = 0;
  for (int d = 0; d < t.ndim; ++d) {
    if (t.sizes[d] == 0) return Extent{};
    const int64_t s = t.strides[d] * (t.sizes[d] - 1);
    if (s < 0) lo += s; else hi += s;
  }
  const uint64_t base = reinterpret_cast<uint64_t>(t.data);
  const int e = esz(t.dtype);
  return Extent{base + (uint64_t)(lo * e), base + (uint64_t)((hi + 1) * e)};
}

// torch broadcasting of `t` onto the output shape: right-aligned, size-1
// dims repeat with stride 0 (fill_tensorref, gpuos_ext.cpp:147-165, does the
// alignment but keeps the input's own sizes; here the strides alone carry it).
void broadcast_to(const gpuos_tensor& t, const gpuos_tensor& out, int64_t* st, const char* what) {
  const int nd = out.ndim;
  for (int d = 0; d < t.ndim - nd; ++d)
    if (t.sizes[d] != 1)
      throw GError(GPUOS_EINVAL, std::string(what) + ": has more dims than the output");
  for (int d = 0; d < nd; ++d) {
    const int od = nd - 1 - d, id = t.ndim - 1 - d;
    const int64_t s_in = id >= 0 ? t.sizes[id] : 1;
    const int64_t str = id >= 0 ? t.strides[id] : 0;
    if (s_in == out.sizes[od]) st[od] = (s_in == 1) ? 0 : str;
    else if (s_in == 1) st[od] = 0;
    else
      throw GError(GPUOS_EINVAL, std::string(what) + ": size " + std::to_string(s_in) +
                                     " does not broadcast to " + std::to_string(out.sizes[od]));
  }
}

double env_double(const char* name, double dflt) {
  const char* v = std::getenv(name);
  if (!v || !*v) return dflt;
  return std::atof(v);
}

}  // namespace

// ---------------------------------------------------------------------------
// helpers
// ---------------------------------------------------------------------------
uint32_t fdiv_magic(uint32_t d, uint32_t* shift) {
  uint32_t s = 0;
  while ((1ull << s) < d) ++s;
  *shift = s;
  return (uint32_t)((((1ull << 32) * ((1ull << s) - d)) / d) + 1);
}

bool IntervalSet::overlaps(const Extent& e) const {
  if (e.empty() || v_.empty()) return false;
  if (e.hi <= v_.front().lo || e.lo >= v_.back().hi) return false;
  // first extent whose hi is above e.lo: the only candidate below e.hi
  size_t lo = 0, hi = v_.size();
  while (lo < hi) {
    const size_t mid = (lo + hi) >> 1;
    if (v_[mid].hi <= e.lo) lo = mid + 1; else hi = mid;
  }
  return lo < v_.size() && v_[lo].lo < e.hi;
}

void IntervalSet::add(Extent e) {
  if (e.empty()) return;
  if (v_.empty() || e.lo > v_.back().hi) {
    v_.push_back(e);
    return;
  }
  if (e.lo >= v_.back().lo) {  // touches or overlaps the last extent only
    if (e.hi > v_.back().hi) v_.back().hi = e.hi;
    return;
  }
  // merge with every extent in [first with hi >= e.lo, last with lo <= e.hi]
  size_t lo = 0, hi = v_.size();
  while (lo < hi) {
    const size_t mid = (lo + hi) >> 1;
    if (v_[mid].hi < e.lo) lo = mid + 1; else hi = mid;
  }
  size_t end = lo;
  while (end < v_.size() && v_[end].lo <= e.hi) {
    e.lo = std::min(e.lo, v_[end].lo);
    e.hi = std::max(e.hi, v_[end].hi);
    ++end;
  }
  if (end == lo) {
    v_.insert(v_.begin() + (ptrdiff_t)lo, e);
  } else {
    v_[lo] = e;
    v_.erase(v_.begin() + (ptrdiff_t)lo + 1, v_.begin() + (ptrdiff_t)end);
  }
}

bool RingAlloc::alloc(uint64_t size, uint64_t tag, uint64_t* off) {
  if (size == 0) { *off = 0; return true; }
  if (size > cap_) return false;
  if (live_.empty()) {
    *off = 0;
    live_.push_back({0, size, tag});
    return true;
  }
  const uint64_t head = live_.front().off;
  const uint64_t tail = live_.back().off + live_.back().size;
  if (tail > head || (tail == head && false)) {
    // [head, tail) in use, free: [tail, cap) and [0, head)
    if (cap_ - tail >= size) { *off = tail; live_.push_back({tail, size, tag}); return true; }
    if (head >= size) { *off = 0; live_.push_back({0, size, tag}); return true; }
    return false;
  }
  // wrapped: in use [head, cap) and [0, tail), free [tail, head)
  if (head - tail >= size) { *off = tail; live_.push_back({tail, size, tag}); return true; }
  return false;
}

void RingAlloc::free_before(uint64_t upto) {
  while (!live_.empty() && live_.front().tag < upto) live_.pop_front();
}

// Relative time per element of an operator's vector body, from per-chunk
// timings of a mixed batch on B200 (light operators 1): a chunk of operator v
// gets 1/chunk_weight(v) of the light operators' elements, so that chunks of
// every operator take about the same time and a batch's slowest warp is not
// the one that drew two transcendental chunks.  The weight-2 operators also
// run the 2-group vector body (op_unroll).
int chunk_weight(int v) {
  switch (v) {
    case V_POW:
      return 8;
    case V_SIGMOID: case V_LOG: case V_SIN: case V_COS: case V_SOFTPLUS:
      return 4;
    case V_TANH: case V_EXP: case V_GELU: case V_ELU: case V_DIV: case V_DIV0: case V_SQRT:
    case V_HARDSWISH:
      return 2;
    default:
      return v >= V_JIT_BASE ? 4 : 1;
  }
}

// Operator names accepted by gpuos_variant_by_name (and the Python layer).
int variant_by_name(const std::string& n) {
  static const std::unordered_map<std::string, int> m = {
      {"add", V_ADD}, {"mul", V_MUL}, {"sub", V_SUB}, {"div0", V_DIV0}, {"batch_div", V_DIV0},
      {"div", V_DIV}, {"maximum", V_MAX}, {"minimum", V_MIN}, {"pow", V_POW}, {"relu", V_RELU},
      {"sigmoid", V_SIGMOID}, {"tanh", V_TANH}, {"exp", V_EXP}, {"log", V_LOG},
      {"sqrt", V_SQRT}, {"abs", V_ABS}, {"hardsigmoid", V_HARDSIGMOID},
      {"hardswish", V_HARDSWISH}, {"gelu", V_GELU}, {"sin", V_SIN}, {"cos", V_COS},
      {"leaky_relu", V_LEAKY_RELU}, {"clamp", V_CLAMP}, {"hardtanh", V_CLAMP}, {"elu", V_ELU},
      {"softplus", V_SOFTPLUS}, {"clamp_min", V_CLAMP_MIN}, {"clamp_max", V_CLAMP_MAX},
      {"copy", V_COPY}, {"sum", V_SUM}, {"mean", V_MEAN}};
  auto it = m.find(n);
  return it == m.end() ? -1 : it->second;
}

// The expression strings the reference scheduler registers
// (pytorch_ext/scheduler.py:145-153, 192-205, 244-290), whitespace removed,
// '#' standing for a float literal with an 'f' suffix.
namespace {
struct ExprPat {
  const char* pat;
  int variant;
  int arity;
};
const ExprPat kExprPats[] = {
    {"(A+B)", V_ADD, 2},
    {"(A-B)", V_SUB, 2},
    {"(A*B)", V_MUL, 2},
    {"(A/B)", V_DIV, 2},
    {"(A>B?A:B)", V_MAX, 2},
    {"(A<B?A:B)", V_MIN, 2},
    {"powf(A,B)", V_POW, 2},
    {"(A>0.f?A:0.f)", V_RELU, 1},
    {"1.f/(1.f+expf(-A))", V_SIGMOID, 1},
    {"tanhf(A)", V_TANH, 1},
    {"expf(A)", V_EXP, 1},
    {"logf(A)", V_LOG, 1},
    {"sqrtf(A)", V_SQRT, 1},
    {"fabsf(A)", V_ABS, 1},
    {"fminf(fmaxf(0.2f*A+0.5f,0.f),1.f)", V_HARDSIGMOID, 1},
    {"A*fminf(fmaxf(A/6.f+0.5f,0.f),1.f)", V_HARDSWISH, 1},
    {"0.5f*A*(1.f+tanhf(0.79788456f*(A+0.044715f*A*A*A)))", V_GELU, 1},
    {"sinf(A)", V_SIN, 1},
    {"cosf(A)", V_COS, 1},
    {"(A>=0.f?A:#*A)", V_LEAKY_RELU, 1},
    {"fminf(fmaxf(A,#),#)", V_CLAMP, 1},
    {"(A>0.f?A:#*(expf(A)-1.f))", V_ELU, 1},
    {"(log1pf(expf(#*A))/#)", V_SOFTPLUS, 1},
    {"fmaxf(A,#)", V_CLAMP_MIN, 1},
    {"fminf(A,#)", V_CLAMP_MAX, 1},
    {"A", V_COPY, 1},
    {"(A)", V_COPY, 1},
};

// parse a C float literal with an 'f' suffix at s[i]; returns chars consumed
size_t parse_flit(const std::string& s, size_t i, float* out) {
  size_t j = i;
  if (j < s.size() && (s[j] == '+' || s[j] == '-')) ++j;
  size_t digits = 0;
  while (j < s.size() && std::isdigit((unsigned char)s[j])) { ++j; ++digits; }
  if (j < s.size() && s[j] == '.') {
    ++j;
    while (j < s.size() && std::isdigit((unsigned char)s[j])) { ++j; ++digits; }
  }
  if (digits == 0) return 0;
  if (j < s.size() && (s[j] == 'e' || s[j] == 'E')) {
    size_t k = j + 1;
    if (k < s.size() && (s[k] == '+' || s[k] == '-')) ++k;
    size_t ed = 0;
    while (k < s.size() && std::isdigit((unsigned char)s[k])) { ++k; ++ed; }
    if (ed == 0) return 0;
    j = k;
  }
  if (j >= s.size() || s[j] != 'f') return 0;
  *out = std::strtof(s.substr(i, j - i).c_str(), nullptr);
  return j + 1 - i;
}
}  // namespace

int match_builtin_expr(const std::string& expr, int arity, float* p0, float* p1) {
  std::string e;
  for (char c : expr)
    if (!std::isspace((unsigned char)c)) e.push_back(c);
  for (const ExprPat& p : kExprPats) {
    if (p.arity != arity) continue;
    const std::string pat = p.pat;
    float vals[2] = {0.f, 0.f};
    int nv = 0;
    size_t i = 0, j = 0;
    bool ok = true;
    while (ok && j < pat.size()) {
      if (pat[j] == '#') {
        float v = 0.f;
        const size_t n = parse_flit(e, i, &v);
        if (n == 0 || nv >= 2) { ok = false; break; }
        vals[nv++] = v;
        i += n;
        ++j;
      } else if (i < e.size() && e[i] == pat[j]) {
        ++i;
        ++j;
      } else {
        ok = false;
      }
    }
    if (!ok || i != e.size()) continue;
    if (p.variant == V_SOFTPLUS && vals[0] != vals[1]) continue;
    *p0 = vals[0];
    *p1 = vals[1];
    return p.variant;
  }
  return -1;
}

// ---------------------------------------------------------------------------
// Executor
// ---------------------------------------------------------------------------
namespace {
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};
}  // namespace

Executor::Executor(int device, const gpuos_options& opt) : device_(device), opt_(opt) {
  DeviceGuard g(device);
  if (opt_.capacity <= 0) opt_.capacity = 4096;
  if (opt_.threads_per_block <= 0) opt_.threads_per_block = 256;
  if (opt_.max_batch <= 0) opt_.max_batch = (int)env_double("GPUOS_BATCH_SHARD", 512);
  opt_.max_batch = std::min(opt_.max_batch, kMaxReqPerBatch);
  if (opt_.mode != GPUOS_MODE_STREAM) opt_.mode = GPUOS_MODE_PERSISTENT;
  int tpb = opt_.threads_per_block;
  if (tpb % 32 != 0 || tpb < 64 || tpb > 1024)
    throw GError(GPUOS_EINVAL, "threads_per_block must be a multiple of 32 in [64, 1024]");
  double idle_ms = opt_.idle_ms > 0 ? opt_.idle_ms : env_double("GPUOS_IDLE_MS", 100.0);
  idle_ms = std::min(std::max(idle_ms, 1.0), 60000.0);
  idle_ns_ = (uint64_t)(idle_ms * 1e6);
  sync_timeout_s_ = opt_.sync_timeout_s > 0 ? opt_.sync_timeout_s
                                            : env_double("GPUOS_SYNC_TIMEOUT_S", 60.0);
  // every wait inside a kernel gives up after this long and reports an error
  wait_limit_ns_ = opt_.wait_limit_us > 0
                       ? (uint64_t)opt_.wait_limit_us * 1000ull
                       : (uint64_t)(std::min(std::max(sync_timeout_s_, 1.0), 10.0) * 1e9);

  GCU(cudaFree(nullptr));
  GCU(cudaDeviceGetAttribute(&sm_count_, cudaDevAttrMultiProcessorCount, device));
  // The CTA shape is fixed by the kernels (eight warps); threads_per_block is
  // accepted for API compatibility.
  block_ = gpuos_cta_threads();
  int bbps = 0, wbps = 0;
  int ebps = 0, rbps = 0;
  GCU(gpuos_occupancy(&bbps, &wbps, &ebps, &rbps));
  ew_bps_ = std::max(1, ebps);
  red_bps_ = std::max(1, rbps);
  if (bbps < 1 || wbps < 2) throw GError(GPUOS_ECUDA, "batch CTAs cannot be resident");
  batch_bps_ = bbps;
  // the persistent grid is fully resident: CTA 0 stages batches, the rest run them
  grid_ = sm_count_ * wbps;
  const int ctas = opt_.mode == GPUOS_MODE_PERSISTENT ? grid_ - 1 : sm_count_ * batch_bps_;
  total_warps_ = ctas * gpuos_cta_threads() / 32;
  lean_grid_ = sm_count_;
  lean_on_ = env_double("GPUOS_LEAN", 1.0) != 0.0;
  chain_on_ = env_double("GPUOS_CHAIN", 1.0) != 0.0;
  lean_warps_ = sm_count_ * kLeanThreads / 32;
  lean_buf_.resize(std::max(gpuos_lean_params_size(2), gpuos_lean_params_size(3)));

  GCU(cudaStreamCreateWithFlags(&s_worker_, cudaStreamNonBlocking));
  GCU(cudaStreamCreateWithFlags(&s_ctrl_, cudaStreamNonBlocking));
  GCU(cudaStreamCreateWithFlags(&s_own_, cudaStreamNonBlocking));
  GCU(cudaStreamCreateWithFlags(&s_copy_, cudaStreamNonBlocking));
  GCU(cudaEventCreateWithFlags(&last_event_, cudaEventDisableTiming));

  // staging arena (pinned, mapped) and its device mirror
  arena_bytes_ = align_up(std::max<uint64_t>(16ull << 20, (uint64_t)opt_.capacity * 1024), 1 << 20);
  GCU(cudaHostAlloc(reinterpret_cast<void**>(&arena_), arena_bytes_, cudaHostAllocMapped));
  GCU(cudaHostGetDevicePointer(reinterpret_cast<void**>(&arena_dev_), arena_, 0));
  GCU(cudaMalloc(reinterpret_cast<void**>(&ring_), arena_bytes_));
  // per-batch counters (self-cleaning; zero before first use)
  GCU(cudaMalloc(reinterpret_cast<void**>(&states_), sizeof(BatchState) * kDoneRing));
  GCU(cudaMemset(states_, 0, sizeof(BatchState) * kDoneRing));
  arena_alloc_.init(arena_bytes_);

  // host control block + rings
  const size_t hb = align_up(sizeof(HostCtrl), 256) + align_up(sizeof(Pub) * kDoneRing, 256) +
                    3 * sizeof(uint64_t) * kDoneRing + 256;
  GCU(cudaHostAlloc(reinterpret_cast<void**>(&hostblk_), hb, cudaHostAllocMapped));
  std::memset(hostblk_, 0, hb);
  GCU(cudaHostGetDevicePointer(reinterpret_cast<void**>(&hostblk_dev_), hostblk_, 0));
  size_t o = 0;
  hctrl_ = reinterpret_cast<HostCtrl*>(hostblk_ + o);
  o += align_up(sizeof(HostCtrl), 256);
  pub_ = reinterpret_cast<Pub*>(hostblk_ + o);
  o += align_up(sizeof(Pub) * kDoneRing, 256);
  done_ring_ = reinterpret_cast<volatile uint64_t*>(hostblk_ + o);
  o += sizeof(uint64_t) * kDoneRing;
  retired_ring_ = reinterpret_cast<volatile uint64_t*>(hostblk_ + o);
  o += sizeof(uint64_t) * kDoneRing;
  dur_ring_ = reinterpret_cast<volatile uint64_t*>(hostblk_ + o);
  o += sizeof(uint64_t) * kDoneRing;
  stop_src_ = hostblk_ + o;
  *reinterpret_cast<uint64_t*>(hostblk_ + o) = UINT64_MAX;  // source of the stop_at reset

  GCU(cudaMalloc(reinterpret_cast<void**>(&dctrl_), sizeof(DevCtrl)));
  GCU(cudaMemset(dctrl_, 0, sizeof(DevCtrl)));

  // jump table: identity alias, slot 0 = add, slot 1 = mul as the reference's
  // init_builtin_ops (persistent_kernel.cu:115-130); slot 10 is the batch
  // operator there and stays reserved here.
  for (int i = 0; i < kMaxSlots; ++i) {
    tab_.alias[i] = i;
    tab_.slot[i] = SlotEntry{V_NONE, 0.f, 0.f, 0};
  }
  tab_.slot[0] = SlotEntry{V_ADD, 0.f, 0.f, 2};
  tab_.slot[1] = SlotEntry{V_MUL, 0.f, 0.f, 2};
  GCU(cudaMalloc(reinterpret_cast<void**>(&dtab_), sizeof(Tables)));
  GCU(cudaMemcpy(dtab_, &tab_, sizeof(Tables), cudaMemcpyHostToDevice));
  // the memsets above ran on the legacy stream; a device-wide synchronisation
  // would also wait for another executor's persistent worker on this device
  GCU(cudaStreamSynchronize(nullptr));
  started_ = true;
  if (opt_.mode == GPUOS_MODE_PERSISTENT) launch_worker_locked(0);
}

Executor::~Executor() {
  try {
    shutdown();
  } catch (...) {
  }
}

void Executor::ensure_scratch_locked() {
  if (partials_) return;
  DeviceGuard g(device_);
  partials_cap_ = 16ull << 20;  // floats
  counters_cap_ = 4ull << 20;   // u32
  GCU(cudaMalloc(reinterpret_cast<void**>(&partials_), partials_cap_ * sizeof(float)));
  GCU(cudaMalloc(reinterpret_cast<void**>(&counters_), counters_cap_ * sizeof(uint32_t)));
  // on the executor's own stream: a device-wide synchronisation would wait
  // for the persistent worker
  GCU(cudaMemsetAsync(counters_, 0, counters_cap_ * sizeof(uint32_t), s_ctrl_));
  GCU(cudaStreamSynchronize(s_ctrl_));
  part_alloc_.init(partials_cap_);
  cnt_alloc_.init(counters_cap_);
}

// ---- request building -----------------------------------------------------
void build_ew(Pending& p, int op, bool is_slot, float p0, float p1,
                        const gpuos_tensor* a, const gpuos_tensor* b, const gpuos_tensor& out) {
  if (!a) throw GError(GPUOS_EINVAL, "input A is required");
  check_tensor(*a, "input A");
  if (b) check_tensor(*b, "input B");
  check_tensor(out, "output");
  const int nd = out.ndim;
  int64_t sa[kMaxDims] = {0}, sb[kMaxDims] = {0};
  broadcast_to(*a, out, sa, "input A");
  if (b) broadcast_to(*b, out, sb, "input B");
  const int64_t numel = numel_of(out);

  struct Dim { int64_t n, a, b, o; };
  Dim dims[kMaxDims];
  int k = 0;
  for (int d = 0; d < nd; ++d)
    if (out.sizes[d] != 1) dims[k++] = Dim{out.sizes[d], sa[d], sb[d], out.strides[d]};
  Dim cd[kMaxDims];
  int m = 0;
  for (int i = 0; i < k; ++i) {
    const Dim& x = dims[i];
    if (m > 0 && cd[m - 1].a == x.a * x.n && cd[m - 1].b == x.b * x.n && cd[m - 1].o == x.o * x.n) {
      cd[m - 1] = Dim{cd[m - 1].n * x.n, x.a, x.b, x.o};
    } else {
      cd[m++] = x;
    }
  }

  Req& q = p.r;
  std::memset(&q, 0, sizeof(q));
  q.op = (uint16_t)op;
  q.kind = RK_EW;
  q.dta = (uint8_t)a->dtype;
  q.dtb = (uint8_t)(b ? b->dtype : a->dtype);
  q.dto = (uint8_t)out.dtype;
  q.flags = (uint8_t)((b ? RF_HAS_B : 0) | (is_slot ? RF_SLOT : 0));
  q.p0 = p0;
  q.p1 = p1;
  q.numel = numel;
  q.a = reinterpret_cast<uint64_t>(a->data);
  q.b = b ? reinterpret_cast<uint64_t>(b->data) : 0;
  q.o = reinterpret_cast<uint64_t>(out.data);
  const int ea = esz(a->dtype), eb = b ? esz(b->dtype) : 0, eo = esz(out.dtype);

  bool a_sc = m > 0, b_sc = b != nullptr && m > 0;
  for (int i = 0; i < m; ++i) {
    if (cd[i].a != 0) a_sc = false;
    if (cd[i].b != 0) b_sc = false;
  }
  auto al4 = [](uint64_t x, int e) { return (x % (uint64_t)(4 * e)) == 0; };

  if (m <= 1 && (m == 0 || cd[0].o == 1) &&
      (m == 0 || cd[0].a == 0 || cd[0].a == 1) &&
      (!b || m == 0 || cd[0].b == 0 || cd[0].b == 1)) {
    q.layout = EL_CONTIG;
    if (a_sc) q.flags |= RF_A_SCALAR;
    if (b_sc) q.flags |= RF_B_SCALAR;
    // vector path: every vector operand aligned to 4 of its elements
    const bool vec = al4(q.o, eo) && (a_sc || al4(q.a, ea)) && (!b || b_sc || al4(q.b, eb));
    if (vec) q.flags |= RF_VEC;
  } else if (m <= 2 && cd[m - 1].o == 1) {
    const int64_t R = (m == 2) ? cd[0].n : 1, N = cd[m - 1].n;
    q.layout = EL_ROW2D;
    q.inner = N;
    q.sa_row = m == 2 ? cd[0].a : 0;
    q.sb_row = m == 2 ? cd[0].b : 0;
    q.so_row = m == 2 ? cd[0].o : 0;
    q.sa_in = cd[m - 1].a;
    q.sb_in = cd[m - 1].b;
    if (a_sc) q.flags |= RF_A_SCALAR;
    if (b_sc) q.flags |= RF_B_SCALAR;
    // vector path: inner size a multiple of 4, every operand either a per-row
    // value (inner stride 0) or 4-aligned rows of unit inner stride
    auto opnd_vec = [&](bool sc, uint64_t ptr, int64_t srow, int64_t sin, int e) {
      if (sc || sin == 0) return true;
      if (sin != 1) return false;
      return al4(ptr, e) && (R == 1 || srow % 4 == 0);
    };
    const bool vec = (N % 4 == 0) && opnd_vec(false, q.o, q.so_row, 1, eo) &&
                     opnd_vec(a_sc, q.a, q.sa_row, q.sa_in, ea) &&
                     (!b || opnd_vec(b_sc, q.b, q.sb_row, q.sb_in, eb));
    if (vec) q.flags |= RF_VEC;
    if (!vec && m == 2 && R <= 1024 && numel < (1ll << 31)) {
      // 2-D tiles: chunks of whole columns, no division per element
      q.layout = EL_TILE2D;
      q.nseg = (uint32_t)R;
    }
    if (numel >= (1ll << 31) || N >= (1ll << 31)) {
      q.flags |= RF_BIG;
    } else {
      uint32_t s = 0;
      q.fdiv_m = fdiv_magic((uint32_t)N, &s);
      q.fdiv_s = s;
    }
  } else {
    q.layout = EL_STRIDED;
    p.has_ext = true;
    std::memset(&p.ext, 0, sizeof(p.ext));
    p.ext.ndim = m;
    for (int i = 0; i < m; ++i) {
      p.ext.sizes[i] = cd[i].n;
      p.ext.sa[i] = cd[i].a;
      p.ext.sb[i] = cd[i].b;
      p.ext.so[i] = cd[i].o;
    }
  }
  // provisional chunking; publish() resizes elementwise chunks per batch
  const uint32_t ce = 2048u;
  q.chunk = ce;
  p.nchunk = (uint32_t)((numel + ce - 1) / ce);
  p.out_ext = extent_of(out);
  p.in_ext[0] = extent_of(*a);
  p.nin = 1;
  if (b) {
    p.in_ext[1] = extent_of(*b);
    p.nin = 2;
  }
}

// A custom expression of three or four operands (RF_NARY): A and B in the
// record, C and D in the extension record.  The general body runs it
// (contiguous, [rows, inner] or up to 8 strided dims after broadcasting and
// dim coalescing), without the vector or 2-D tile paths.
void build_ew_nary(Pending& p, int op, bool is_slot, float p0, float p1,
                   const gpuos_tensor* const* ins, int nin, const gpuos_tensor& out) {
  static const char* names[4] = {"input A", "input B", "input C", "input D"};
  if (nin < 3 || nin > 4) throw GError(GPUOS_EINVAL, "a request takes 1 to 4 inputs");
  for (int k = 0; k < nin; ++k) {
    if (!ins[k]) throw GError(GPUOS_EINVAL, std::string(names[k]) + " is required");
    check_tensor(*ins[k], names[k]);
  }
  check_tensor(out, "output");
  const int nd = out.ndim;
  int64_t st[4][kMaxDims] = {};
  for (int k = 0; k < nin; ++k) broadcast_to(*ins[k], out, st[k], names[k]);
  const int64_t numel = numel_of(out);

  struct Dim { int64_t n, s[4], o; };
  Dim dims[kMaxDims];
  int kd = 0;
  for (int d = 0; d < nd; ++d)
    if (out.sizes[d] != 1) {
      Dim x{out.sizes[d], {0, 0, 0, 0}, out.strides[d]};
      for (int k = 0; k < nin; ++k) x.s[k] = st[k][d];
      dims[kd++] = x;
    }
  Dim cd[kMaxDims];
  int m = 0;
  for (int i = 0; i < kd; ++i) {
    const Dim& x = dims[i];
    bool merge = m > 0 && cd[m - 1].o == x.o * x.n;
    for (int k = 0; k < nin && merge; ++k) merge = cd[m - 1].s[k] == x.s[k] * x.n;
    if (merge) {
      Dim y = x;
      y.n = cd[m - 1].n * x.n;
      cd[m - 1] = y;
    } else {
      cd[m++] = x;
    }
  }

  Req& q = p.r;
  std::memset(&q, 0, sizeof(q));
  q.op = (uint16_t)op;
  q.kind = RK_EW;
  q.dta = (uint8_t)ins[0]->dtype;
  q.dtb = (uint8_t)ins[1]->dtype;
  q.dto = (uint8_t)out.dtype;
  q.flags = (uint8_t)(RF_HAS_B | RF_NARY | (is_slot ? RF_SLOT : 0));
  q.p0 = p0;
  q.p1 = p1;
  q.numel = numel;
  q.a = reinterpret_cast<uint64_t>(ins[0]->data);
  q.b = reinterpret_cast<uint64_t>(ins[1]->data);
  q.o = reinterpret_cast<uint64_t>(out.data);
  p.has_ext = true;
  std::memset(&p.ext, 0, sizeof(p.ext));
  p.ext.c = reinterpret_cast<uint64_t>(ins[2]->data);
  p.ext.dtc = ins[2]->dtype;
  p.ext.d = nin > 3 ? reinterpret_cast<uint64_t>(ins[3]->data) : 0;
  p.ext.dtd = nin > 3 ? ins[3]->dtype : ins[2]->dtype;

  bool unit = m <= 1 && (m == 0 || cd[0].o == 1);
  for (int k = 0; k < nin && unit && m == 1; ++k) unit = cd[0].s[k] == 0 || cd[0].s[k] == 1;
  if (unit) {
    q.layout = EL_CONTIG;
    if (m == 0 || cd[0].s[0] == 0) q.flags |= RF_A_SCALAR;
    if (m == 0 || cd[0].s[1] == 0) q.flags |= RF_B_SCALAR;
    p.ext.sc[0] = m ? cd[0].s[2] : 0;
    p.ext.sd[0] = (m && nin > 3) ? cd[0].s[3] : 0;
  } else if (m <= 2 && cd[m - 1].o == 1) {
    const int64_t N = cd[m - 1].n;
    q.layout = EL_ROW2D;
    q.inner = N;
    q.sa_row = m == 2 ? cd[0].s[0] : 0;
    q.sb_row = m == 2 ? cd[0].s[1] : 0;
    q.so_row = m == 2 ? cd[0].o : 0;
    q.sa_in = cd[m - 1].s[0];
    q.sb_in = cd[m - 1].s[1];
    p.ext.sc[0] = m == 2 ? cd[0].s[2] : 0;
    p.ext.sc[1] = cd[m - 1].s[2];
    p.ext.sd[0] = (m == 2 && nin > 3) ? cd[0].s[3] : 0;
    p.ext.sd[1] = nin > 3 ? cd[m - 1].s[3] : 0;
    if (numel >= (1ll << 31) || N >= (1ll << 31)) {
      q.flags |= RF_BIG;
    } else {
      uint32_t sh = 0;
      q.fdiv_m = fdiv_magic((uint32_t)N, &sh);
      q.fdiv_s = sh;
    }
  } else {
    q.layout = EL_STRIDED;
    p.ext.ndim = m;
    for (int i = 0; i < m; ++i) {
      p.ext.sizes[i] = cd[i].n;
      p.ext.sa[i] = cd[i].s[0];
      p.ext.sb[i] = cd[i].s[1];
      p.ext.sc[i] = cd[i].s[2];
      p.ext.sd[i] = nin > 3 ? cd[i].s[3] : 0;
      p.ext.so[i] = cd[i].o;
    }
  }
  const uint32_t ce = 2048u;
  q.chunk = ce;
  p.nchunk = (uint32_t)((numel + ce - 1) / ce);
  p.out_ext = extent_of(out);
  for (int k = 0; k < nin; ++k) p.in_ext[k] = extent_of(*ins[k]);
  p.nin = nin;
}

void build_reduce(Pending& p, int op, bool is_slot, const gpuos_tensor& x,
                            const gpuos_tensor& out, const int32_t* axes, int naxes,
                            bool keepdim) {
  check_tensor(x, "input");
  check_tensor(out, "output");
  const int nd = x.ndim;
  bool red[kMaxDims] = {false};
  int nred = 0;
  for (int i = 0; i < naxes; ++i) {
    int ax = axes[i];
    if (ax < 0) ax += nd;
    if (ax < 0 || ax >= nd) throw GError(GPUOS_EINVAL, "reduction axis out of range");
    if (!red[ax]) { red[ax] = true; ++nred; }
  }
  const int out_nd = keepdim ? nd : nd - nred;
  if (out.ndim != out_nd)
    throw GError(GPUOS_EINVAL, "output has " + std::to_string(out.ndim) + " dims, expected " +
                                   std::to_string(out_nd));
  struct KD { int64_t n, sa, so; };
  struct RD { int64_t n, s; };
  KD kd[kMaxDims];
  RD rd[kMaxDims];
  int nk = 0, nr = 0, od = 0;
  int64_t C = 1;
  for (int d = 0; d < nd; ++d) {
    if (red[d]) {
      if (keepdim) {
        if (out.sizes[od] != 1) throw GError(GPUOS_EINVAL, "keepdim output must have size 1 on reduced axes");
        ++od;
      }
      C *= x.sizes[d];
      if (x.sizes[d] != 1) rd[nr++] = RD{x.sizes[d], x.strides[d]};
    } else {
      if (out.sizes[od] != x.sizes[d]) throw GError(GPUOS_EINVAL, "output shape does not match input");
      if (x.sizes[d] != 1) kd[nk++] = KD{x.sizes[d], x.strides[d], out.strides[od]};
      ++od;
    }
  }
  // coalesce kept dims (input and output strides together) and reduced dims
  KD ck[kMaxDims];
  RD cr[kMaxDims];
  int mk = 0, mr = 0;
  for (int i = 0; i < nk; ++i) {
    if (mk > 0 && ck[mk - 1].sa == kd[i].sa * kd[i].n && ck[mk - 1].so == kd[i].so * kd[i].n)
      ck[mk - 1] = KD{ck[mk - 1].n * kd[i].n, kd[i].sa, kd[i].so};
    else
      ck[mk++] = kd[i];
  }
  for (int i = 0; i < nr; ++i) {
    if (mr > 0 && cr[mr - 1].s == rd[i].s * rd[i].n)
      cr[mr - 1] = RD{cr[mr - 1].n * rd[i].n, rd[i].s};
    else
      cr[mr++] = rd[i];
  }
  const int64_t R = numel_of(out);

  Req& q = p.r;
  std::memset(&q, 0, sizeof(q));
  q.op = (uint16_t)op;
  q.kind = RK_RED;
  q.dta = (uint8_t)x.dtype;
  q.dtb = (uint8_t)x.dtype;
  q.dto = (uint8_t)out.dtype;
  q.flags = (uint8_t)(is_slot ? RF_SLOT : 0);
  q.numel = R;
  q.inner = C;
  q.a = reinterpret_cast<uint64_t>(x.data);
  q.o = reinterpret_cast<uint64_t>(out.data);
  q.nseg = 1;
  const int e = esz(x.dtype);
  // elements per chunk (or per segment of a long row): 64 KB of input
  // (measured on the reduction stream: 0.575 of HBM against 0.549 with 32 KB)
  const int64_t kSeg = 65536 / e;

  if (mk <= 1 && mr <= 1) {
    const int64_t sr = mk ? ck[0].sa : 0, so = mk ? ck[0].so : 0;
    const int64_t sc = mr ? cr[0].s : 1;
    q.sa_row = sr;
    q.so_row = so;
    q.sa_in = sc;
    if (sc == 1) {
      q.layout = RL_ROWS;
      // rows are read in aligned 16-byte blocks, whatever their alignment
      q.flags |= RF_VEC;
      if (C <= kSeg) {
        // lanes per row: as many as leave each lane at most 8 of the 16-byte
        // blocks a row touches, so that a row step is one round of loads
        const uint64_t nbl = (uint64_t)(C * e + 15) / 16 + 1;
        const uint32_t G = std::min<uint32_t>(32, pow2_ceil((nbl + 7) / 8));
        const uint32_t per = 32 / G;
        uint64_t rpc = (uint64_t)std::max<int64_t>(1, kSeg / std::max<int64_t>(C, 1));
        rpc = std::max<uint64_t>(per, rpc / per * per);
        q.rg = G;
        q.chunk = (uint32_t)rpc;
        p.nchunk = (uint32_t)((R + (int64_t)rpc - 1) / (int64_t)rpc);
      } else {
        q.rg = 32;
        q.chunk = (uint32_t)kSeg;
        q.nseg = (uint32_t)((C + kSeg - 1) / kSeg);
        p.nchunk = (uint32_t)(R * q.nseg);
        p.partials = (uint64_t)R * q.nseg;
        p.counters = (uint64_t)R;
      }
    } else if (sr == 1 && mk <= 1 && mr == 1 && (q.a & 15) == 0 && ((sc * e) & 15) == 0 &&
               R % (16 / e) == 0 && R >= 16 * (16 / e)) {
      // rows adjacent, 16-byte aligned: each lane reads 16 bytes of adjacent
      // rows per column (red_cols_vec); chunks of 32 x GE rows by `chunk` columns
      q.layout = RL_COLS;
      q.flags |= RF_VEC;
      const int64_t GE = 16 / e;
      const uint32_t rg = (uint32_t)(32 * GE);
      // about 8192 elements a chunk, as a contiguous row chunk holds
      int64_t seglen = std::max<int64_t>(8, kSeg / rg);
      int64_t nseg = std::max<int64_t>(1, (C + seglen - 1) / seglen);
      if (nseg > 256) {
        seglen = (C + 255) / 256;
        nseg = (C + seglen - 1) / seglen;
      }
      const int64_t ngroups = (R + rg - 1) / rg;
      q.rg = rg;
      q.chunk = (uint32_t)seglen;
      q.nseg = (uint32_t)nseg;
      p.nchunk = (uint32_t)(ngroups * nseg);
      if (nseg > 1) {
        p.partials = (uint64_t)(ngroups * nseg * rg);
        p.counters = (uint64_t)ngroups;
      }
    } else {
      q.layout = RL_COLS;
      const uint32_t rg = std::min<uint32_t>(32, pow2_ceil((uint64_t)std::max<int64_t>(R, 1)));
      const uint32_t cl = 32 / rg;
      int64_t seglen = std::max<int64_t>(cl, kSeg / rg);
      int64_t nseg = std::max<int64_t>(1, (C + seglen - 1) / seglen);
      if (nseg > 256) {
        seglen = align_up((uint64_t)((C + 255) / 256), cl);
        nseg = (C + seglen - 1) / seglen;
      }
      const int64_t ngroups = (R + rg - 1) / rg;
      q.rg = rg;
      q.chunk = (uint32_t)seglen;
      q.nseg = (uint32_t)nseg;
      p.nchunk = (uint32_t)(ngroups * nseg);
      if (nseg > 1) {
        p.partials = (uint64_t)(ngroups * nseg * rg);
        p.counters = (uint64_t)ngroups;
      }
    }
  } else {
    q.layout = RL_GENERIC;
    if (C >= 64) {
      // a warp per output (red_generic_warp), a few outputs per chunk
      q.rg = 1;
      q.chunk = (uint32_t)std::max<int64_t>(1, kSeg / C);
    } else {
      // a lane per output (red_generic), 32 outputs per chunk
      q.chunk = 32;
    }
    p.nchunk = (uint32_t)((R + q.chunk - 1) / q.chunk);
    p.has_ext = true;
    std::memset(&p.ext, 0, sizeof(p.ext));
    p.ext.ndim = mk;
    p.ext.rdim = mr;
    for (int i = 0; i < mk; ++i) {
      p.ext.sizes[i] = ck[i].n;
      p.ext.sa[i] = ck[i].sa;
      p.ext.so[i] = ck[i].so;
    }
    for (int i = 0; i < mr; ++i) {
      p.ext.rsizes[i] = cr[i].n;
      p.ext.rstrides[i] = cr[i].s;
    }
  }
  if ((uint64_t)p.nchunk * 1 > 0xffffffffull) throw GError(GPUOS_EINVAL, "request too large");
  p.out_ext = extent_of(out);
  p.in_ext[0] = extent_of(x);
  p.nin = 1;
}

void Executor::submit_ew(int op, bool is_slot, float p0, float p1, const gpuos_tensor* a,
                         const gpuos_tensor* b, const gpuos_tensor& out) {
  std::lock_guard<std::mutex> lk(mu_);
  if (!started_) throw GError(GPUOS_ESTATE, "executor is shut down");
  // planned in place: a Pending is large (it can hold a strided layout)
  pending_.emplace_back();
  try {
    build_ew(pending_.back(), op, is_slot, p0, p1, a, b, out);
  } catch (...) {
    pending_.pop_back();
    throw;
  }
  ++requests_;
  if (pending_.back().nchunk == 0) pending_.pop_back();  // empty output: nothing to do
}

void Executor::submit_nary(int slot, const gpuos_tensor* const* ins, int nin,
                           const gpuos_tensor& out) {
  std::lock_guard<std::mutex> lk(mu_);
  if (!started_) throw GError(GPUOS_ESTATE, "executor is shut down");
  if (slot < 0 || slot >= kMaxSlots) throw GError(GPUOS_EINVAL, "slot out of range");
  const int phys = tab_.alias[slot];
  const SlotEntry& e = tab_.slot[phys >= 0 && phys < kMaxSlots ? phys : slot];
  if (e.arity != nin)
    throw GError(GPUOS_EINVAL, "slot " + std::to_string(slot) + " takes " +
                                   std::to_string(e.arity) + " inputs, got " +
                                   std::to_string(nin));
  pending_.emplace_back();
  try {
    build_ew_nary(pending_.back(), slot, true, 0.f, 0.f, ins, nin, out);
  } catch (...) {
    pending_.pop_back();
    throw;
  }
  ++requests_;
  if (pending_.back().nchunk == 0) pending_.pop_back();
}

void Executor::submit_reduce(int op, bool is_slot, const gpuos_tensor& x,
                             const gpuos_tensor& out, const int32_t* axes, int naxes,
                             bool keepdim) {
  Pending p;
  build_reduce(p, op, is_slot, x, out, axes, naxes, keepdim);
  std::lock_guard<std::mutex> lk(mu_);
  if (!started_) throw GError(GPUOS_ESTATE, "executor is shut down");
  ++requests_;
  if (p.nchunk == 0) return;
  pending_.push_back(p);
}

// The reference's Task (src/common.h:34-46), accepted as-is.
namespace {
struct RefTensorRef {
  void* data;
  int32_t dtype;
  int32_t ndim;
  int64_t sizes[8];
  int64_t strides[8];
};
struct RefTask {
  int32_t op, flags, ndim;
  int64_t numel;
  int32_t rrank;
  int32_t r_axes[8];
  int32_t r_keepdim;
  RefTensorRef in0, in1, out0;
};
static_assert(sizeof(RefTensorRef) == 144, "TensorRef layout");
static_assert(sizeof(RefTask) == 496, "Task layout");
static_assert(offsetof(RefTask, numel) == 16 && offsetof(RefTask, rrank) == 24 &&
                  offsetof(RefTask, in0) == 64 && offsetof(RefTask, in1) == 208 &&
                  offsetof(RefTask, out0) == 352,
              "Task field offsets");
static_assert(sizeof(RefTensorRef) == sizeof(gpuos_tensor), "gpuos_tensor mirrors TensorRef");
}  // namespace

void Executor::submit_task(const void* task) {
  RefTask t;
  std::memcpy(&t, task, sizeof(t));
  if (t.op == 10)
    throw GError(GPUOS_EINVAL, "slot 10 is the batch operator; batches are built by gpuos_flush");
  gpuos_tensor in0, in1, out0;
  std::memcpy(&in0, &t.in0, sizeof(in0));
  std::memcpy(&in1, &t.in1, sizeof(in1));
  std::memcpy(&out0, &t.out0, sizeof(out0));
  if (t.rrank > 0) {
    if (t.rrank > 8) throw GError(GPUOS_EINVAL, "rrank > 8");
    submit_reduce(t.op, true, in0, out0, t.r_axes, t.rrank, t.r_keepdim != 0);
  } else {
    submit_ew(t.op, true, 0.f, 0.f, &in0, t.in1.data ? &in1 : nullptr, out0);
  }
}

// ---- batches ----------------------------------------------------------------
void Executor::reclaim() {
  if (opt_.mode == GPUOS_MODE_STREAM) {
    // a batch is done once the event recorded after its launch has completed;
    // the kernel posts a completion word only for a batch with errors
    while (done_wm_ < next_seq_) {
      uint32_t e = 0;
      if (lean_seq_[done_wm_ % kDoneRing]) {
        // a lean batch posts seq + 1 when its last CTA is done
        const uint64_t w = done_ring_[done_wm_ % kDoneRing];
        if ((w & kDoneMask) != done_wm_ + 1) break;
        e = (uint32_t)((w >> 48) & 0xffu);
        if (e) {
          ++errors_;
          if (err_seq_ == UINT64_MAX) err_seq_ = done_wm_;
          err_bits_ |= e;
        }
        dev_ns_ += dur_ring_[done_wm_ % kDoneRing];
        ++done_wm_;
        continue;
      }
      const cudaError_t q = cudaEventQuery(done_ev_[done_wm_ % kDoneRing]);
      if (q == cudaErrorNotReady) break;
      if (q != cudaSuccess) {
        e = ERR_CUDA;
        if (cuda_err_.empty()) cuda_err_ = cudaGetErrorString(q);
      } else {
        const uint64_t w = done_ring_[done_wm_ % kDoneRing];
        e = (w & kDoneMask) == done_wm_ + 1 ? (uint32_t)((w >> 48) & 0xffu) : 0u;
        if (e) e |= take_batch_err(done_wm_);
      }
      if (e) {
        ++errors_;
        if (err_seq_ == UINT64_MAX) err_seq_ = done_wm_;
        err_bits_ |= e;
      }
      ++done_wm_;
    }
    retired_wm_ = done_wm_;
  }
  while (done_wm_ < next_seq_) {
    const uint64_t w = done_ring_[done_wm_ % kDoneRing];
    if ((w & kDoneMask) != done_wm_ + 1) break;
    const uint32_t e = (uint32_t)((w >> 48) & 0xffu);
    if (e) {
      ++errors_;
      if (err_seq_ == UINT64_MAX) err_seq_ = done_wm_;
      err_bits_ |= e;
    }
    dev_ns_ += dur_ring_[done_wm_ % kDoneRing];
    ++done_wm_;
  }
  while (retired_wm_ < next_seq_) {
    if (retired_ring_[retired_wm_ % kDoneRing] != retired_wm_ + 1) break;
    ++retired_wm_;
  }
  arena_alloc_.free_before(retired_wm_);
  part_alloc_.free_before(retired_wm_);
  cnt_alloc_.free_before(retired_wm_);
  if (done_wm_ == next_seq_) {
    live_out_.clear();
    live_in_.clear();
  }
}

// A stream-mode batch that posted an error word itself (no end-of-batch
// protocol ran): its complete error bits are in its device counters; read
// them and clear the slot for its next use.  Only runs for failed batches.
uint32_t Executor::take_batch_err(uint64_t seq) {
  DeviceGuard g(device_);
  BatchState st;
  std::memset(&st, 0, sizeof(st));
  BatchState* d = states_ + seq % kDoneRing;
  if (cudaMemcpyAsync(&st, d, sizeof(st), cudaMemcpyDeviceToHost, s_ctrl_) != cudaSuccess ||
      cudaMemsetAsync(d, 0, sizeof(st), s_ctrl_) != cudaSuccess ||
      cudaStreamSynchronize(s_ctrl_) != cudaSuccess) {
    if (cuda_err_.empty()) cuda_err_ = "reading a failed batch's error bits";
    return ERR_CUDA;
  }
  return st.err;
}

bool Executor::wait_for_room_locked(std::unique_lock<std::mutex>& lk, uint64_t bytes,
                                    uint64_t floats, uint64_t counters, uint64_t* arena_off,
                                    uint64_t* part_off, uint64_t* cnt_off, uint64_t seq) {
  const auto t0 = std::chrono::steady_clock::now();
  for (int it = 0;; ++it) {
    reclaim();
    if (next_seq_ - retired_wm_ < (uint64_t)kDoneRing - 1) {
      uint64_t ao = 0, po = 0, co = 0;
      if (arena_alloc_.alloc(bytes, seq, &ao)) {
        const bool pok = floats == 0 || part_alloc_.alloc(floats, seq, &po);
        const bool cok = pok && (counters == 0 || cnt_alloc_.alloc(counters, seq, &co));
        if (pok && cok) {
          *arena_off = ao;
          *part_off = po;
          *cnt_off = co;
          return true;
        }
        // give back what this attempt took and wait for older batches to retire
        if (pok && floats) part_alloc_.undo_last();
        arena_alloc_.undo_last();
      }
    }
    if (opt_.mode == GPUOS_MODE_PERSISTENT) ensure_worker_locked();
    const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > sync_timeout_s_) return false;
    lk.unlock();
    if (it < 64) GPUOS_PAUSE();
    else if (it < 512) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(20));
    lk.lock();
  }
}

void Executor::publish(std::unique_lock<std::mutex>& lk, std::vector<Pending>& reqs, size_t i,
                       size_t j, cudaStream_t stream) {
  const uint32_t n = (uint32_t)(j - i);
  // hazards between the requests of this batch: a request that reads what an
  // earlier request of its stage writes (or writes what it reads or writes)
  // opens a new stage; chunks of a stage start after the previous stage is done.
  std::vector<uint32_t> stage_first(n, 0u);
  IntervalSet so, si;
  uint32_t cur = 0;
  bool staged = false, after_prev = false;
  bool check_live = opt_.mode == GPUOS_MODE_PERSISTENT && done_wm_ < next_seq_;
  // Fast path, one pass: outputs that follow one another in address order
  // without overlap, and inputs whose hull no output touches, have no hazard
  // (the usual shape of a stream of requests on slab-allocated tensors).
  bool fast = true;
  Extent oh{UINT64_MAX, 0}, ih{UINT64_MAX, 0};
  uint64_t prev_hi = 0;
  for (uint32_t r = 0; r < n && fast; ++r) {
    const Pending& p = reqs[i + r];
    if (!p.out_ext.empty()) {
      if (p.out_ext.lo < prev_hi) fast = false;
      prev_hi = p.out_ext.hi;
      oh.lo = std::min(oh.lo, p.out_ext.lo);
      oh.hi = std::max(oh.hi, p.out_ext.hi);
    }
    for (int k = 0; k < p.nin; ++k) {
      if (p.in_ext[k].empty()) continue;
      ih.lo = std::min(ih.lo, p.in_ext[k].lo);
      ih.hi = std::max(ih.hi, p.in_ext[k].hi);
    }
  }
  auto meets = [](const Extent& a, const Extent& b) {
    return !a.empty() && !b.empty() && a.lo < b.hi && b.lo < a.hi;
  };
  if (fast && meets(oh, ih)) fast = false;
  if (fast && check_live) {
    // and none of the batches in flight writes what this one touches, or
    // reads what it writes
    const Extent lo_h = live_out_.hull(), li_h = live_in_.hull();
    if (!meets(oh, lo_h) && !meets(ih, lo_h) && !meets(oh, li_h)) check_live = false;
  }
  for (uint32_t r = 0; r < n && (!fast || check_live); ++r) {
    const Pending& p = reqs[i + r];
    if (!fast) {
      bool hz = so.overlaps(p.out_ext) || si.overlaps(p.out_ext);
      for (int k = 0; k < p.nin && !hz; ++k) hz = so.overlaps(p.in_ext[k]);
      if (hz) {
        so.clear();
        si.clear();
        cur = r;
        staged = true;
      }
      stage_first[r] = cur;
      so.add(p.out_ext);
      for (int k = 0; k < p.nin; ++k) si.add(p.in_ext[k]);
    }
    if (check_live && !after_prev) {
      bool lz = live_out_.overlaps(p.out_ext) || live_in_.overlaps(p.out_ext);
      for (int k = 0; k < p.nin && !lz; ++k) lz = live_out_.overlaps(p.in_ext[k]);
      after_prev = lz;
    }
  }
  // Time per element of a request's chunks, in units of half a light
  // operator's fp32 vector element: the operator's weight, times 2 for the
  // vector body with per-row operands and 4 for the general body (from
  // per-chunk timings).  (Counting 16-bit vector elements at half measured
  // slower on the broadcast stream: their chunks are not cheaper per element.)
  auto ew_cost = [](const Pending& p, int v) -> uint64_t {
    uint64_t w = 2 * (uint64_t)chunk_weight(v);
    const bool vec = (p.r.flags & RF_VEC) && p.r.layout != EL_STRIDED;
    if (p.r.layout == EL_TILE2D) w *= 2;
    else if (!vec) w *= 4;
    else if (p.r.layout == EL_ROW2D) w *= 2;
    return w;
  };
  // Elementwise chunk size for this batch: about two light-operator chunks'
  // worth of work per resident warp, as a multiple of 512 elements in
  // 512..8192 of a light fp32 operator,
  // counting each element at its cost; a request's chunks get 1/cost of that
  // (at least 128 elements).
  std::vector<int> var(n);
  std::vector<uint8_t> cost_log2(n);  // every cost is a power of two
  uint64_t ew_work = 0, est_bytes = 0;
  for (uint32_t r = 0; r < n; ++r) {
    Pending& p = reqs[i + r];
    int v = p.r.op;
    if (p.r.flags & RF_SLOT) {
      const int s = p.r.op;
      const int phys = (s >= 0 && s < kMaxSlots) ? tab_.alias[s] : -1;
      v = (phys >= 0 && phys < kMaxSlots) ? tab_.slot[phys].variant : V_NONE;
    }
    var[r] = v;
    if (p.r.kind == RK_EW) {
      cost_log2[r] = (uint8_t)__builtin_ctzll(ew_cost(p, v));
      ew_work += (uint64_t)p.r.numel << cost_log2[r];
      est_bytes += (uint64_t)p.r.numel * 12u;
    } else {
      est_bytes += (uint64_t)p.r.numel * (uint64_t)p.r.inner * 4u;
    }
  }
  // a lean batch: the whole batch in the lean kernel's parameters (lean.cuh)
  bool lean = lean_on_ && opt_.mode == GPUOS_MODE_STREAM && !staged && n <= (uint32_t)kLeanUniMax;
  for (uint32_t r = 0; r < n && lean; ++r) lean = lean_eligible(reqs[i + r], var[r]);
  if (lean) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    GCU(cudaStreamIsCapturing(stream, &cap));
    lean = cap == cudaStreamCaptureStatusNone;
  }
  const uint64_t warps = lean ? (uint64_t)std::max(1, lean_warps_)
                              : (uint64_t)std::max(1, total_warps_);
  uint64_t ce = align_up(std::max<uint64_t>(1, ew_work / (2 * warps)), 1024);
  ce = std::min<uint64_t>(std::max<uint64_t>(ce, 1024), 16384);
  // A batch with stage barriers runs its stages one after another, each on
  // as many warps as it has chunks: a stage's chunks are sized from its own
  // work spread over every warp (one chunk per granule, below), not from the
  // whole batch's.
  std::vector<uint64_t> stage_ce;
  if (staged) {
    std::vector<uint64_t> sw(n, 0);
    for (uint32_t r = 0; r < n; ++r)
      // (elementwise work only: reduction chunks are sized per request, by
      // build_reduce, whatever else shares their stage)
      if (reqs[i + r].r.kind == RK_EW) sw[stage_first[r]] += (uint64_t)reqs[i + r].r.numel << cost_log2[r];
    stage_ce.resize(n);
    for (uint32_t r = 0; r < n; ++r) {
      const uint64_t c = align_up(std::max<uint64_t>(1, sw[stage_first[r]] / warps), 256);
      stage_ce[r] = std::min<uint64_t>(std::max<uint64_t>(c, 1024), 16384);
    }
  }
  for (uint32_t r = 0; r < n; ++r) {
    Pending& p = reqs[i + r];
    if (p.r.kind != RK_EW) continue;
    uint64_t c = std::max<uint64_t>(128, (staged ? stage_ce[r] : ce) >> cost_log2[r]);
    if (p.r.layout == EL_TILE2D) {
      // whole columns: c elements make c / rows columns, a multiple of the
      // 32 x kTileC columns a warp covers per pass (64)
      const uint64_t R = std::max<uint32_t>(1u, p.r.nseg), N = (uint64_t)p.r.inner;
      uint64_t cols = align_up(std::max<uint64_t>(1, c / R), 64);
      const uint64_t k = (N + cols - 1) / cols;
      cols = align_up((N + k - 1) / k, 64);
      p.r.chunk = (uint32_t)cols;
      p.nchunk = (uint32_t)((N + cols - 1) / cols);
      continue;
    }
    if (p.r.layout == EL_STRIDED) c = std::min<uint64_t>(c, 2048);
    // equal chunks (a multiple of 4 elements, as the vector path needs)
    const uint64_t numel = (uint64_t)p.r.numel;
    const uint64_t k = (numel + c - 1) / c;
    c = align_up((numel + k - 1) / k, 4);
    p.r.chunk = (uint32_t)c;
    p.nchunk = (uint32_t)((numel + c - 1) / c);
  }
  // Within each stage the order of requests is free: group them by operator
  // so that the warps of an SM run few operator bodies at a time.
  // (a stable counting sort on a 256-entry key: kind and variant)
  std::vector<uint32_t> order(n);
  {
    auto key = [&](uint32_t r) -> uint32_t {
      return ((uint32_t)reqs[i + r].r.kind << 7) | ((uint32_t)var[r] & 127u);
    };
    uint32_t counts[257];
    for (uint32_t s0 = 0; s0 < n;) {
      uint32_t s1 = s0 + 1;
      while (s1 < n && stage_first[s1] == stage_first[s0]) ++s1;
      std::memset(counts, 0, sizeof(counts));
      for (uint32_t r = s0; r < s1; ++r) ++counts[key(r) + 1];
      for (int b = 0; b < 256; ++b) counts[b + 1] += counts[b];
      for (uint32_t r = s0; r < s1; ++r) order[s0 + counts[key(r)]++] = r;
      s0 = s1;
    }
  }
  if (lean) {
    uint64_t lchunks = 0;
    for (uint32_t r = 0; r < n; ++r) lchunks += reqs[i + r].nchunk;
    if (publish_lean(lk, reqs, i, n, var, order, lchunks, stream)) return;
  }
  if (opt_.mode == GPUOS_MODE_STREAM) {
    // a batch that is not lean runs after everything before it on the stream
    lean_prev_in_flush_ = false;
    lean_out_.clear();
    lean_in_.clear();
  }
  // payload layout
  std::vector<uint32_t> cb(n + 1);
  uint64_t nchunk = 0, floats = 0, counters = 0;
  uint32_t next = 0;
  for (uint32_t r = 0; r < n; ++r) {
    const Pending& p = reqs[i + order[r]];
    cb[r] = (uint32_t)nchunk;
    nchunk += p.nchunk;
    floats += p.partials;
    counters += p.counters;
    if (p.has_ext) ++next;
  }
  cb[n] = (uint32_t)nchunk;
  if (nchunk > 0xffffffffull) throw GError(GPUOS_EINVAL, "batch too large");
  // Granules: the unit of work a warp takes at a time, about eight per warp
  // (at most 8 chunks each): chunks of different requests cost different
  // times, and more granules per warp even out the warps' totals.
  // (a batch with stage barriers: one chunk each, so that a stage spreads
  // over as many warps as it has chunks)
  const uint64_t warps_all = (uint64_t)std::max(1, total_warps_);
  uint64_t gran = staged ? 1 : nchunk / (8 * warps_all);
  gran = std::min<uint64_t>(std::max<uint64_t>(gran, 1), 8);
  // A batch of at least 16 chunks per warp (the large reductions) has its
  // warps claim granules one at a time, so that chunks of different costs
  // (dtypes, layouts) even out across warps; at that size the claims (one
  // atomic per granule of up to 8 chunks) are noise.
  const bool claim = !staged && nchunk >= 16 * warps_all;
  // claimed granules small enough for about 32 claims per warp: the last
  // granule a warp claims is the batch's tail
  if (claim) gran = std::min<uint64_t>(std::max<uint64_t>(nchunk / (32 * warps_all), 1), 8);
  const uint64_t ngran = (nchunk + gran - 1) / gran;
  const uint64_t rec_off = sizeof(BatchHdr);
  const uint64_t cb_off = rec_off + 128ull * n;
  // the granule table is read as 8-byte pairs
  const uint64_t gtab_off = align_up(cb_off + 4ull * (n + 1), 8);
  const uint64_t wait_off = gtab_off + 8ull * ngran;
  const uint64_t ext_off = align_up(wait_off + (staged ? 4ull * n : 0), 16);
  const uint64_t bytes = align_up(ext_off + sizeof(ExtRec) * (uint64_t)next, 16);
  if (floats || counters) ensure_scratch_locked();
  if (bytes > arena_bytes_ || floats > partials_cap_ || counters > counters_cap_)
    throw GError(GPUOS_EINVAL, "batch does not fit the staging memory");

  const uint64_t seq = next_seq_;
  uint64_t aoff = 0, poff = 0, coff = 0;
  if (!wait_for_room_locked(lk, bytes, floats, counters, &aoff, &poff, &coff, seq))
    throw GError(GPUOS_ETIMEOUT, "timed out waiting for staging memory");
  uint8_t* base = arena_ + aoff;
  std::memset(base, 0, sizeof(BatchHdr));
  BatchHdr* h = reinterpret_cast<BatchHdr*>(base);
  h->seq = seq;
  h->nreq = n;
  h->nchunk = (uint32_t)nchunk;
  h->rec_off = (uint32_t)rec_off;
  h->cb_off = (uint32_t)cb_off;
  h->bytes = (uint32_t)bytes;
  h->flags = (staged ? BF_STAGED : 0u) | (after_prev ? BF_AFTER_PREV : 0u) |
             (claim ? BF_CLAIM : 0u);
  h->scratch = floats ? reinterpret_cast<uint64_t>(partials_ + poff) : 0;
  h->counters = reinterpret_cast<uint64_t>(counters_);
  h->wait_from = done_wm_;
  h->gtab_off = (uint32_t)gtab_off;
  h->gran = (uint32_t)gran;
  Req* recs = reinterpret_cast<Req*>(base + rec_off);
  uint32_t* cbp = reinterpret_cast<uint32_t*>(base + cb_off);
  ExtRec* ext = reinterpret_cast<ExtRec*>(base + ext_off);
  uint64_t pf = 0, pc = coff, xi = 0;
  // a batch with a custom expression runs in the kernel linked with them,
  // which has every precompiled body as well
  bool jit_batch = false;
  for (uint32_t r = 0; r < n && !jit_batch; ++r) jit_batch = var[r] >= V_JIT_BASE;
  // the persistent worker resolves slot requests itself, from its copy of the
  // jump table, when it starts them
  const bool dev_resolve = opt_.mode == GPUOS_MODE_PERSISTENT && !jit_batch;
  for (uint32_t r = 0; r < n; ++r) {
    Pending& p = reqs[i + order[r]];
    Req q = p.r;
    // otherwise the operator (and parameters) the request's slot names now:
    // the device runs the record as it stands
    if ((q.flags & RF_SLOT) && !dev_resolve) {
      const int s = q.op;
      const int phys = (s >= 0 && s < kMaxSlots) ? tab_.alias[s] : -1;
      if (phys >= 0 && phys < kMaxSlots) {
        q.p0 = tab_.slot[phys].p0;
        q.p1 = tab_.slot[phys].p1;
      }
      q.flags = (uint8_t)(q.flags & ~RF_SLOT);
    }
    if (!(q.flags & RF_SLOT)) q.op = var[order[r]] < 0 ? kOpNone : (uint16_t)var[order[r]];
    if (p.has_ext) {
      ext[xi] = p.ext;
      q.ext = (uint32_t)(ext_off + sizeof(ExtRec) * xi);
      ++xi;
    }
    if (p.partials) {
      q.part = (uint32_t)pf;
      pf += p.partials;
    }
    if (p.counters) {
      q.cnt = (uint32_t)pc;
      pc += p.counters;
    }
    recs[r] = q;
  }
  std::memcpy(cbp, cb.data(), 4ull * (n + 1));
  {
    // granule j starts at chunk j * gran, inside the request whose chunks
    // [cb[r], cb[r + 1]) hold it: walk the requests once
    uint32_t* gt = reinterpret_cast<uint32_t*>(base + gtab_off);
    uint64_t j = 0;
    for (uint32_t r = 0; r < n && j < ngran; ++r) {
      const uint64_t end = cb[r + 1];
      for (uint64_t c = j * gran; c < end; c = ++j * gran) {
        gt[2 * j] = r;
        gt[2 * j + 1] = cb[r];
      }
    }
  }
  bool stalled = false;
  if (staged) {
    uint32_t* w = reinterpret_cast<uint32_t*>(base + wait_off);
    for (uint32_t r = 0; r < n; ++r) w[r] = stage_first[r] ? cb[stage_first[r]] : 0u;
    if (stall_next_) {
      // fault injection: the last stage waits for one chunk more than the
      // earlier stages have, which only its own (waiting) chunks could add
      // (on the polled stage barriers: such a batch does not run as a chain)
      stall_next_ = false;
      stalled = true;
      const uint32_t last = stage_first[n - 1];
      for (uint32_t r = 0; r < n; ++r)
        if (stage_first[order[r]] == last) w[r] = cb[last] + 1u;
    }
  }
  if (jit_batch && opt_.mode == GPUOS_MODE_PERSISTENT) {
    // Custom expressions do not run in the resident worker: the batch runs
    // after every earlier batch, on its own launch, before any later one.  It
    // takes no sequence number; its staging memory is freed with the next
    // batch's.
    run_jit_batch_sync_locked(lk, aoff, bytes, ngran, h);
    return;
  }
  next_seq_ = seq + 1;

  if (opt_.mode == GPUOS_MODE_PERSISTENT) {
    dur_ring_[seq % kDoneRing] = 0;
    Pub& pb = pub_[seq % kDoneRing];
    pb.seq = seq;
    pb.off = (uint32_t)aoff;
    pb.bytes = (uint32_t)bytes;
    std::atomic_thread_fence(std::memory_order_seq_cst);
    hctrl_->tail = seq + 1;
    std::atomic_thread_fence(std::memory_order_seq_cst);
    for (uint32_t r = 0; r < n; ++r) {
      live_out_.add(reqs[i + r].out_ext);
      for (int k = 0; k < reqs[i + r].nin; ++k) live_in_.add(reqs[i + r].in_ext[k]);
    }
    ensure_worker_locked();
  } else {
    DeviceGuard g(device_);
    if (have_last_stream_ && stream != last_stream_ && done_wm_ < seq) {
      GCU(cudaEventRecord(last_event_, last_stream_));
      GCU(cudaStreamWaitEvent(stream, last_event_, 0));
    }
    // The payload is copied on the executor's copy stream, which the launch
    // waits on: the copy runs while the caller's stream is still busy with
    // earlier work, instead of in front of this kernel.  (Its ring space was
    // freed only after the kernel that used it before had completed.)  A
    // stream being captured into a graph copies in line.
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    GCU(cudaStreamIsCapturing(stream, &cap));
    if (cap == cudaStreamCaptureStatusNone) {
      cudaEvent_t& ce = copy_ev_[seq % kDoneRing];
      if (!ce) GCU(cudaEventCreateWithFlags(&ce, cudaEventDisableTiming));
      GCU(cudaMemcpyAsync(ring_ + aoff, arena_ + aoff, bytes, cudaMemcpyHostToDevice, s_copy_));
      GCU(cudaEventRecord(ce, s_copy_));
      GCU(cudaStreamWaitEvent(stream, ce, 0));
    } else {
      GCU(cudaMemcpyAsync(ring_ + aoff, arena_ + aoff, bytes, cudaMemcpyHostToDevice, stream));
    }
    // a batch of one class of requests runs the kernel with only those bodies
    int bodies = 0;
    for (uint32_t r = 0; r < n; ++r) bodies |= reqs[i + r].r.kind == RK_EW ? 1 : 2;
    const int bps = bodies == 1 ? ew_bps_ : bodies == 2 ? red_bps_ : batch_bps_;
    const uint64_t wpc = (uint64_t)block_ / 32;
    int grid = (int)std::min<uint64_t>((uint64_t)sm_count_ * (jit_batch ? batch_bps_ : bps),
                                       (ngran + wpc - 1) / wpc);
    grid = std::max(grid, 1);
    volatile uint64_t* dr = reinterpret_cast<volatile uint64_t*>(
        hostblk_dev_ + (reinterpret_cast<const volatile uint8_t*>(done_ring_) - hostblk_));
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (timing_) {
      for (cudaEvent_t* e : {&e0, &e1}) {
        if (ev_pool_.empty()) {
          GCU(cudaEventCreate(e));
        } else {
          *e = ev_pool_.back();
          ev_pool_.pop_back();
        }
      }
      GCU(cudaEventRecord(e0, stream));
    }
    // A small batch with stage barriers (at most 32 MB, counting 12 bytes an
    // elementwise element and 4 a reduced one) runs on one cluster of 8 CTAs
    // with cluster barriers between its stages (chain_batch).
    const bool chain = staged && !stalled && !jit_batch && chain_on_ && est_bytes <= (32ull << 20);
    if (jit_batch) {
      jit_launch(jit_kernels_.back(), grid, block_, stream, ring_ + aoff, *h,
                 states_ + seq % kDoneRing, dr, wait_limit_ns_);
    } else if (chain) {
      GCU(gpuos_launch_chain(ring_ + aoff, h, states_ + seq % kDoneRing, dr, wait_limit_ns_, 8,
                             stream));
      ++chain_count_;
    } else {
      GCU(gpuos_launch_batch(ring_ + aoff, h, states_ + seq % kDoneRing, dr, wait_limit_ns_, grid,
                             stream, bodies));
    }
    if (timing_) {
      GCU(cudaEventRecord(e1, stream));
      timed_.emplace_back(e0, e1);
    }
    // completion (and the reuse of the batch's staging memory) is this event
    lean_seq_[seq % kDoneRing] = 0;
    cudaEvent_t& de = done_ev_[seq % kDoneRing];
    if (!de) GCU(cudaEventCreateWithFlags(&de, cudaEventDisableTiming));
    GCU(cudaEventRecord(de, stream));
    last_stream_ = stream;
    have_last_stream_ = true;
  }
}

namespace {
bool variant_binary(int v) {
  return v == V_ADD || v == V_MUL || v == V_SUB || v == V_DIV0 || v == V_DIV || v == V_MAX ||
         v == V_MIN || v == V_POW;
}

// (p0, p1) a request runs with: its own, or its slot's when it names a slot
void effective_params(const Tables& tab, const Req& q, float* p0, float* p1) {
  *p0 = q.p0;
  *p1 = q.p1;
  if (q.flags & RF_SLOT) {
    const int s = q.op;
    const int phys = (s >= 0 && s < kMaxSlots) ? tab.alias[s] : -1;
    if (phys >= 0 && phys < kMaxSlots) {
      *p0 = tab.slot[phys].p0;
      *p1 = tab.slot[phys].p1;
    }
  }
}

template <int N>
void fill_lean(uint8_t* buf, uint64_t seq, uint64_t st, uint64_t done_ring, uint64_t dur_ring,
               uint32_t flags,
               const std::vector<Pending>& reqs, size_t i, uint32_t n, const std::vector<int>& var,
               const std::vector<uint32_t>& order, uint64_t nchunk, const Tables& tab) {
  LeanBatch<N>* b = reinterpret_cast<LeanBatch<N>*>(buf);
  std::memset(&b->h, 0, sizeof(b->h));
  b->h.seq = seq;
  b->h.st = st;
  b->h.done_ring = done_ring;
  b->h.dur_ring = dur_ring;
  b->h.nreq = n;
  b->h.nchunk = (uint32_t)nchunk;
  b->h.flags = flags;
  int npar = 0;
  uint32_t c = 0;
  for (uint32_t r = 0; r < n; ++r) {
    const Pending& p = reqs[i + order[r]];
    float p0, p1;
    effective_params(tab, p.r, &p0, &p1);
    int k = 0;
    while (k < npar && !(b->h.par[k][0] == p0 && b->h.par[k][1] == p1)) ++k;
    if (k == npar) {
      b->h.par[k][0] = p0;
      b->h.par[k][1] = p1;
      ++npar;
    }
    LeanRec& q = b->rec[r];
    q.a = p.r.a;
    q.b = p.r.b;
    q.o = p.r.o;
    q.numel = (uint32_t)p.r.numel;
    q.chunk = p.r.chunk;
    q.op = (uint8_t)var[order[r]];
    q.flags = (uint8_t)(p.r.flags & RF_HAS_B);
    q.pidx = (uint8_t)k;
    b->cb[r] = c;
    c += p.nchunk;
  }
  b->cb[n] = c;
}
}  // namespace

// A request the lean kernel can run: contiguous, 16-byte aligned fp32 tensors
// (no scalar operands) of a precompiled elementwise operator, with B present
// when the operator reads it.
// The parameter block of a batch of requests of one shape (LeanUniBatch).
void fill_lean_uni(uint8_t* buf, uint64_t seq, uint64_t st, uint64_t done_ring, uint64_t dur_ring,
                   uint32_t flags, const std::vector<Pending>& reqs, size_t i, uint32_t n,
                   const std::vector<int>& var, const std::vector<uint32_t>& order,
                   uint64_t nchunk, const Tables& tab) {
  LeanUniBatch* b = reinterpret_cast<LeanUniBatch*>(buf);
  std::memset(&b->h, 0, sizeof(b->h));
  b->h.seq = seq;
  b->h.st = st;
  b->h.done_ring = done_ring;
  b->h.dur_ring = dur_ring;
  b->h.nreq = n;
  b->h.nchunk = (uint32_t)nchunk;
  b->h.flags = flags;
  const Pending& p0 = reqs[i];
  b->numel = (uint32_t)p0.r.numel;
  b->chunk = p0.r.chunk;
  b->kpr = p0.nchunk;
  b->pad = 0;
  int npar = 0;
  for (uint32_t r = 0; r < n; ++r) {
    const Pending& p = reqs[i + order[r]];
    float p0v, p1v;
    effective_params(tab, p.r, &p0v, &p1v);
    int k = 0;
    while (k < npar && !(b->h.par[k][0] == p0v && b->h.par[k][1] == p1v)) ++k;
    if (k == npar) {
      b->h.par[k][0] = p0v;
      b->h.par[k][1] = p1v;
      ++npar;
    }
    b->a[r] = p.r.a;
    b->b[r] = p.r.b;
    b->o[r] = p.r.o;
    b->op[r] = (uint8_t)var[order[r]];
    b->pidx[r] = (uint8_t)k;
  }
}

bool Executor::lean_eligible(const Pending& p, int v) const {
  const Req& q = p.r;
  if (q.kind != RK_EW || q.layout != EL_CONTIG || !(q.flags & RF_VEC) || p.has_ext) return false;
  if (q.flags & (RF_A_SCALAR | RF_B_SCALAR)) return false;
  if (v < 0 || v >= V_NUM_EW || q.numel >= (1ll << 31)) return false;
  if (q.dta != kF32 || q.dto != kF32) return false;
  const bool hasb = q.flags & RF_HAS_B;
  if (hasb && q.dtb != kF32) return false;
  if (variant_binary(v) && !hasb) return false;
  return true;
}

// Publish one lean batch.  Returns false (nothing published) when its
// parameters do not fit the block (more than kLeanPar distinct pairs).
bool Executor::publish_lean(std::unique_lock<std::mutex>& lk, std::vector<Pending>& reqs,
                            size_t i, uint32_t n, const std::vector<int>& var,
                            const std::vector<uint32_t>& order, uint64_t nchunk,
                            cudaStream_t stream) {
  {
    std::vector<std::pair<float, float>> pars;
    for (uint32_t r = 0; r < n; ++r) {
      float p0, p1;
      effective_params(tab_, reqs[i + r].r, &p0, &p1);
      if (std::find(pars.begin(), pars.end(), std::make_pair(p0, p1)) == pars.end())
        pars.emplace_back(p0, p1);
      if (pars.size() > (size_t)kLeanPar) return false;
    }
  }
  if (nchunk == 0 || nchunk > 0x7fffffffull) return false;
  // more requests than a LeanBatch holds: only as requests of one shape
  bool uni = false;
  if (n > (uint32_t)kLeanMaxReq) {
    const Pending& p0 = reqs[i];
    uni = n <= (uint32_t)kLeanUniMax;
    for (uint32_t r = 1; r < n && uni; ++r) {
      const Pending& p = reqs[i + r];
      uni = p.r.numel == p0.r.numel && p.r.chunk == p0.r.chunk && p.nchunk == p0.nchunk;
    }
    if (!uni) return false;
  }
  // a free batch slot (counters and completion word)
  const auto t0 = std::chrono::steady_clock::now();
  for (int it = 0;; ++it) {
    reclaim();
    if (next_seq_ - retired_wm_ < (uint64_t)kDoneRing - 1) break;
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() >
        sync_timeout_s_)
      throw GError(GPUOS_ETIMEOUT, "timed out waiting for a free batch slot");
    lk.unlock();
    if (it < 64) GPUOS_PAUSE();
    else std::this_thread::sleep_for(std::chrono::microseconds(20));
    lk.lock();
  }
  const uint64_t seq = next_seq_;
  // wait for the previous grid unless it is a lean batch of this flush that
  // shares no memory with this one
  bool wf = !lean_prev_in_flush_;
  for (uint32_t r = 0; r < n && !wf; ++r) {
    const Pending& p = reqs[i + r];
    wf = lean_out_.overlaps(p.out_ext) || lean_in_.overlaps(p.out_ext);
    for (int k = 0; k < p.nin && !wf; ++k) wf = lean_out_.overlaps(p.in_ext[k]);
  }
  const int cls = uni ? 3 : n <= 32 ? 0 : (n <= 128 ? 1 : 2);
  const uint64_t st = reinterpret_cast<uint64_t>(states_ + seq % kDoneRing);
  const uint64_t dr = reinterpret_cast<uint64_t>(
      hostblk_dev_ + (reinterpret_cast<const volatile uint8_t*>(done_ring_) - hostblk_));
  const uint64_t du = reinterpret_cast<uint64_t>(
      hostblk_dev_ + (reinterpret_cast<const volatile uint8_t*>(dur_ring_) - hostblk_));
  const uint32_t flags = wf ? LEAN_WAIT_FIRST : 0u;
  uint8_t* buf = lean_buf_.data();
  if (cls == 0) fill_lean<32>(buf, seq, st, dr, du, flags, reqs, i, n, var, order, nchunk, tab_);
  else if (cls == 1) fill_lean<128>(buf, seq, st, dr, du, flags, reqs, i, n, var, order, nchunk, tab_);
  else if (cls == 2) fill_lean<kLeanMaxReq>(buf, seq, st, dr, du, flags, reqs, i, n, var, order, nchunk, tab_);
  else fill_lean_uni(buf, seq, st, dr, du, flags, reqs, i, n, var, order, nchunk, tab_);
  dur_ring_[seq % kDoneRing] = 0;
  DeviceGuard g(device_);
  if (have_last_stream_ && stream != last_stream_ && done_wm_ < seq) {
    GCU(cudaEventRecord(last_event_, last_stream_));
    GCU(cudaStreamWaitEvent(stream, last_event_, 0));
  }
  const int wpc = kLeanThreads / 32;
  const int grid = (int)std::min<uint64_t>((uint64_t)lean_grid_,
                                           std::max<uint64_t>(1, (nchunk + wpc - 1) / wpc));
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (timing_) {
    for (cudaEvent_t* e : {&e0, &e1}) {
      if (ev_pool_.empty()) {
        GCU(cudaEventCreate(e));
      } else {
        *e = ev_pool_.back();
        ev_pool_.pop_back();
      }
    }
    GCU(cudaEventRecord(e0, stream));
  }
  lean_seq_[seq % kDoneRing] = 1;
  GCU(gpuos_launch_lean(buf, cls, grid, stream));
  if (timing_) {
    GCU(cudaEventRecord(e1, stream));
    timed_.emplace_back(e0, e1);
  }
  next_seq_ = seq + 1;
  ++lean_count_;
  lean_prev_in_flush_ = !timing_;
  for (uint32_t r = 0; r < n; ++r) {
    lean_out_.add(reqs[i + r].out_ext);
    for (int k = 0; k < reqs[i + r].nin; ++k) lean_in_.add(reqs[i + r].in_ext[k]);
  }
  last_stream_ = stream;
  have_last_stream_ = true;
  return true;
}

// The variant a request's record will carry (its slot resolved now).
int Executor::variant_of(const Pending& p) const {
  if (!(p.r.flags & RF_SLOT)) return p.r.op;
  const int s = p.r.op;
  const int phys = (s >= 0 && s < kMaxSlots) ? tab_.alias[s] : -1;
  return (phys >= 0 && phys < kMaxSlots) ? tab_.slot[phys].variant : V_NONE;
}

// Persistent mode: one batch of custom-expression requests, staged at `aoff`
// of the arena, run on the executor's stream once every earlier batch is done.
void Executor::run_jit_batch_sync_locked(std::unique_lock<std::mutex>& lk, uint64_t aoff,
                                         uint64_t bytes, uint64_t ngran, BatchHdr* h) {
  const auto t0 = std::chrono::steady_clock::now();
  for (int it = 0;; ++it) {
    reclaim();
    if (done_wm_ == next_seq_) break;
    ensure_worker_locked();
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() >
        sync_timeout_s_)
      throw GError(GPUOS_ETIMEOUT, "timed out waiting for earlier batches");
    lk.unlock();
    if (it < 64) GPUOS_PAUSE();
    else std::this_thread::sleep_for(std::chrono::microseconds(20));
    lk.lock();
  }
  DeviceGuard g(device_);
  if (worker_launched_) {
    // the resident worker holds the SMs' registers: let it exit first (it is
    // idle); the next batch relaunches it
    hctrl_->quit = 1u;
    std::atomic_thread_fence(std::memory_order_seq_cst);
    const auto t1 = std::chrono::steady_clock::now();
    cudaError_t q;
    while ((q = cudaStreamQuery(s_worker_)) == cudaErrorNotReady) {
      if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t1).count() >
          sync_timeout_s_)
        throw GError(GPUOS_ETIMEOUT, "persistent worker did not exit");
      std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    hctrl_->quit = 0u;
    std::atomic_thread_fence(std::memory_order_seq_cst);
    worker_launched_ = false;
    if (q != cudaSuccess) GCU(q);
  }
  if (!jit_state_) {
    GCU(cudaMalloc(reinterpret_cast<void**>(&jit_state_), sizeof(BatchState)));
    GCU(cudaMemset(jit_state_, 0, sizeof(BatchState)));
    void* w = nullptr;
    GCU(cudaHostAlloc(&w, 64, cudaHostAllocMapped));
    jit_word_ = static_cast<volatile uint64_t*>(w);
  }
  h->seq = 0;  // its error word is jit_word_[0]
  jit_word_[0] = 0;
  void* wd = nullptr;
  GCU(cudaHostGetDevicePointer(&wd, const_cast<uint64_t*>(jit_word_), 0));
  GCU(cudaMemcpyAsync(ring_ + aoff, arena_ + aoff, bytes, cudaMemcpyHostToDevice, s_own_));
  const uint64_t wpc = (uint64_t)block_ / 32;
  int grid = (int)std::min<uint64_t>((uint64_t)sm_count_ * batch_bps_, (ngran + wpc - 1) / wpc);
  jit_launch(jit_kernels_.back(), std::max(grid, 1), block_, s_own_, ring_ + aoff, *h,
             jit_state_, static_cast<volatile uint64_t*>(wd), wait_limit_ns_);
  GCU(cudaStreamSynchronize(s_own_));
  const uint64_t w = jit_word_[0];
  if ((w & kDoneMask) == 1) {
    const uint32_t e = (uint32_t)((w >> 48) & 0xffu);
    if (e) {
      ++errors_;
      throw GError(GPUOS_EDEVICE, "gpuos batch error in a custom-expression batch (bits " +
                                      std::to_string(e) + ")");
    }
  }
}

uint64_t Executor::flush(bool sync, cudaStream_t stream) {
  uint64_t ticket;
  {
    std::unique_lock<std::mutex> lk(mu_);
    if (!started_) throw GError(GPUOS_ESTATE, "executor is shut down");
    std::vector<Pending> reqs;
    reqs.swap(pending_);
    if (!reqs.empty()) {
      DeviceGuard g(device_);
      // stream NULL is CUDA's legacy default stream, as everywhere in CUDA
      if (opt_.mode == GPUOS_MODE_PERSISTENT && stream != s_own_) {
        // the worker reads the inputs as soon as the doorbell rings, so work
        // still queued on the producer stream must finish first
        cudaError_t qs = cudaStreamQuery(stream);
        if (qs == cudaErrorNotReady) GCU(cudaStreamSynchronize(stream));
        else if (qs != cudaSuccess) GCU(qs);
      }
      size_t i = 0;
      const uint64_t budget = arena_bytes_ / 4;
      lean_prev_in_flush_ = false;
      lean_out_.clear();
      lean_in_.clear();
      // stream mode: batches no larger than a lean parameter block holds
      const bool lean_mode = opt_.mode == GPUOS_MODE_STREAM && lean_on_;
      const size_t cap = lean_mode ? std::min<size_t>(opt_.max_batch, kLeanMaxReq)
                                   : (size_t)opt_.max_batch;
      while (i < reqs.size()) {
        size_t j = i;
        uint64_t bytes = 256, floats = 0, cnts = 0, chunks = 0;
        // A run of lean requests of one shape (element count and operator
        // cost class, so one chunk length) fills a batch of up to 1024: its
        // parameter block (LeanUniBatch) holds twice as many requests.
        size_t cap_i = cap;
        if (lean_mode && opt_.max_batch >= kLeanMaxReq) {
          const Pending& p0 = reqs[i];
          const int v0 = variant_of(p0);
          size_t k = i;
          if (lean_eligible(p0, v0))
            while (k < reqs.size() && k - i < (size_t)kLeanUniMax) {
              const Pending& p = reqs[k];
              const int v = variant_of(p);
              if (p.r.numel != p0.r.numel || !lean_eligible(p, v) ||
                  chunk_weight(v) != chunk_weight(v0))
                break;
              ++k;
            }
          if (k - i > cap) cap_i = k - i;
        }
        while (j < reqs.size() && j - i < cap_i) {
          const Pending& p = reqs[j];
          const uint64_t b = 136 + (p.has_ext ? sizeof(ExtRec) : 0);
          if (j > i && (bytes + b > budget || floats + p.partials > (16ull << 20) / 2 ||
                        cnts + p.counters > (4ull << 20) / 2 ||
                        chunks + p.nchunk > 0x7fffffffull))
            break;
          bytes += b;
          floats += p.partials;
          cnts += p.counters;
          chunks += p.nchunk;
          ++j;
        }
        publish(lk, reqs, i, j, stream);
        i = j;
      }
      // hand the vector's capacity back so that the next requests do not regrow it
      reqs.clear();
      if (pending_.empty()) pending_.swap(reqs);
    }
    ticket = next_seq_;
  }
  if (sync) wait(ticket, sync_timeout_s_);
  return ticket;
}

// With mu_ held and every batch before `ticket` done: raise the error of a
// failed batch among them (once).
void Executor::raise_batch_error_locked(uint64_t ticket) {
  if (err_seq_ != UINT64_MAX && err_seq_ < ticket) {
    const uint32_t e = err_bits_;
    err_seq_ = UINT64_MAX;
    err_bits_ = 0;
    std::string why;
    if (e & ERR_BAD_OP) why += " a request used a slot with no registered operator;";
    if (e & ERR_BAD_KIND) why += " a slot's operator does not fit the request kind;";
    if (e & ERR_STAGE_TIMEOUT) why += " a stage barrier wait timed out;";
    if (e & ERR_CUDA) why += " CUDA reported: " + cuda_err_ + ";";
    throw GError(GPUOS_EDEVICE, "gpuos batch error:" + why);
  }
}

bool Executor::poll(uint64_t ticket) {
  std::lock_guard<std::mutex> lk(mu_);
  reclaim();
  if (done_wm_ < ticket) return false;
  raise_batch_error_locked(ticket);
  return true;
}

void Executor::wait(uint64_t ticket, double timeout_s) {
  if (timeout_s <= 0) timeout_s = sync_timeout_s_;
  const auto t0 = std::chrono::steady_clock::now();
  for (int it = 0;; ++it) {
    {
      std::lock_guard<std::mutex> lk(mu_);
      reclaim();
      if (done_wm_ >= ticket) {
        raise_batch_error_locked(ticket);
        return;
      }
      if (opt_.mode == GPUOS_MODE_PERSISTENT) ensure_worker_locked();
      if (opt_.mode == GPUOS_MODE_STREAM && (it & 1023) == 1023 && have_last_stream_) {
        // a lean batch completes through its word only: a kernel that failed
        // never writes it, so look at the stream's error state now and then
        DeviceGuard g(device_);
        const cudaError_t q = cudaStreamQuery(last_stream_);
        if (q != cudaSuccess && q != cudaErrorNotReady)
          throw GError(GPUOS_ECUDA, std::string("the batch stream reported: ") +
                                        cudaGetErrorString(q));
      }
    }
    const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > timeout_s)
      throw GError(GPUOS_ETIMEOUT, "timed out waiting for batch completion (done " +
                                       std::to_string(done_wm_) + " of " +
                                       std::to_string(ticket) + ")");
    if (it < 256) GPUOS_PAUSE();
    else if (it < 4096) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

// ---- persistent worker -----------------------------------------------------
void Executor::launch_worker_locked(uint64_t start) {
  DeviceGuard g(device_);
  hctrl_->running = 1u;
  hctrl_->exit_reason = 0u;
  hctrl_->idle_ns = idle_ns_;
  std::atomic_thread_fence(std::memory_order_seq_cst);
  GCU(cudaMemcpyAsync(&dctrl_->stop_at, stop_src_, sizeof(uint64_t), cudaMemcpyHostToDevice,
                      s_worker_));
  WorkerArgs w;
  w.ring = ring_;
  w.states = states_;
  w.arena = arena_dev_;
  w.hctrl = reinterpret_cast<volatile HostCtrl*>(hostblk_dev_);
  w.pub = reinterpret_cast<const volatile Pub*>(
      hostblk_dev_ + (reinterpret_cast<uint8_t*>(pub_) - hostblk_));
  w.dctrl = dctrl_;
  w.done_ring = reinterpret_cast<volatile uint64_t*>(
      hostblk_dev_ + (reinterpret_cast<const volatile uint8_t*>(done_ring_) - hostblk_));
  w.retired_ring = reinterpret_cast<volatile uint64_t*>(
      hostblk_dev_ + (reinterpret_cast<const volatile uint8_t*>(retired_ring_) - hostblk_));
  w.dur_ring = reinterpret_cast<volatile uint64_t*>(
      hostblk_dev_ + (reinterpret_cast<const volatile uint8_t*>(dur_ring_) - hostblk_));
  w.tab = dtab_;
  w.start_seq = start;
  w.wait_limit_ns = wait_limit_ns_;
  w.idle_ns = idle_ns_;
  GCU(gpuos_launch_worker(&w, grid_, s_worker_));
  worker_launched_ = true;
  ++relaunches_;
}

void Executor::ensure_worker_locked() {
  if (opt_.mode != GPUOS_MODE_PERSISTENT || !started_) return;
  DeviceGuard g(device_);
  if (worker_launched_) {
    cudaError_t q = cudaStreamQuery(s_worker_);
    if (q == cudaErrorNotReady) {
      if (hctrl_->running) return;
      if (hctrl_->staged >= next_seq_) return;
      // stopping while work is pending: let it finish exiting (bounded)
      const auto t0 = std::chrono::steady_clock::now();
      while ((q = cudaStreamQuery(s_worker_)) == cudaErrorNotReady) {
        const double el =
            std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (el > sync_timeout_s_) throw GError(GPUOS_ETIMEOUT, "persistent worker did not exit");
        std::this_thread::yield();
      }
    }
    if (q != cudaSuccess) GCU(q);
    worker_launched_ = false;
  }
  if (hctrl_->staged < next_seq_) launch_worker_locked(hctrl_->staged);
}

bool Executor::worker_alive() {
  std::lock_guard<std::mutex> lk(mu_);
  if (opt_.mode != GPUOS_MODE_PERSISTENT || !started_ || !worker_launched_) return false;
  DeviceGuard g(device_);
  cudaError_t q = cudaStreamQuery(s_worker_);
  if (q == cudaErrorNotReady) return true;
  if (q != cudaSuccess) GCU(q);
  worker_launched_ = false;
  return false;
}

// ---- jump table --------------------------------------------------------------
int Executor::register_elementwise(const std::string& key, const std::string& expr, int arity) {
  std::lock_guard<std::mutex> lk(mu_);
  auto it = slot_of_key_.find(key);
  if (it != slot_of_key_.end()) return it->second;
  if (arity < 1 || arity > 4) throw GError(GPUOS_EINVAL, "arity must be 1 to 4");
  float p0 = 0.f, p1 = 0.f;
  int v = arity <= 2 ? match_builtin_expr(expr, arity, &p0, &p1) : -1;
  if (next_slot_ >= kMaxSlots) throw GError(GPUOS_EINVAL, "jump table is full (128 slots)");
  if (v < 0) {
    // not a precompiled operator: compile it (with the earlier custom ones)
    // and link a new batch kernel
    std::vector<std::string> exprs = jit_exprs_;
    exprs.push_back(expr);
    const std::vector<char> cubin = jit_compile(exprs);
    DeviceGuard g(device_);
    jit_kernels_.push_back(jit_link(cubin));
    jit_exprs_ = exprs;
    v = V_JIT_BASE + (int)jit_exprs_.size() - 1;
  }
  const int slot = next_slot_++;
  tab_.slot[slot] = SlotEntry{v, p0, p1, arity};
  push_tables_locked();
  slot_of_key_.emplace(key, slot);
  return slot;
}

int Executor::register_reduce(const std::string& key, const std::string& op_name) {
  std::lock_guard<std::mutex> lk(mu_);
  auto it = slot_of_key_.find(key);
  if (it != slot_of_key_.end()) return it->second;
  int v;
  if (op_name == "sum") v = V_SUM;
  else if (op_name == "mean") v = V_MEAN;
  else throw GError(GPUOS_EINVAL, "reduce op must be 'sum' or 'mean'");
  if (next_slot_ >= kMaxSlots) throw GError(GPUOS_EINVAL, "jump table is full (128 slots)");
  const int slot = next_slot_++;
  tab_.slot[slot] = SlotEntry{v, 0.f, 0.f, 1};
  push_tables_locked();
  slot_of_key_.emplace(key, slot);
  return slot;
}

void Executor::set_alias(int logical, int physical) {
  if (logical < 0 || logical >= kMaxSlots || physical < 0 || physical >= kMaxSlots)
    throw GError(GPUOS_EINVAL, "slot out of range");
  std::lock_guard<std::mutex> lk(mu_);
  tab_.alias[logical] = physical;
  push_tables_locked();
}

// Publish the jump table to its device copy (the persistent worker reads it
// with acquire loads when it starts a slot request); returns once the copy
// has landed, so a swap is visible to every request the worker starts after
// the call returns.
void Executor::push_tables_locked() {
  DeviceGuard g(device_);
  GCU(cudaMemcpyAsync(dtab_, &tab_, sizeof(Tables), cudaMemcpyHostToDevice, s_ctrl_));
  GCU(cudaStreamSynchronize(s_ctrl_));
}

void Executor::set_slot(int slot, int variant, float p0, float p1) {
  if (slot < 0 || slot >= kMaxSlots) throw GError(GPUOS_EINVAL, "slot out of range");
  const bool ok = variant == V_NONE || (variant >= 0 && variant < V_NUM_EW) ||
                  (variant >= V_JIT_BASE && variant < V_JIT_BASE + (int)jit_exprs_.size()) ||
                  variant == V_SUM || variant == V_MEAN;
  if (!ok) throw GError(GPUOS_EINVAL, "unknown operator id " + std::to_string(variant));
  std::lock_guard<std::mutex> lk(mu_);
  const int arity = (variant == V_ADD || variant == V_MUL || variant == V_SUB ||
                     variant == V_DIV0 || variant == V_DIV || variant == V_MAX ||
                     variant == V_MIN || variant == V_POW) ? 2 : 1;
  tab_.slot[slot] = SlotEntry{variant, p0, p1, arity};
  push_tables_locked();
}

void Executor::get_slot(int slot, int* variant, float* p0, float* p1, int* alias) {
  if (slot < 0 || slot >= kMaxSlots) throw GError(GPUOS_EINVAL, "slot out of range");
  std::lock_guard<std::mutex> lk(mu_);
  if (variant) *variant = tab_.slot[slot].variant;
  if (p0) *p0 = tab_.slot[slot].p0;
  if (p1) *p1 = tab_.slot[slot].p1;
  if (alias) *alias = tab_.alias[slot];
}

void Executor::set_timing(bool on) {
  std::lock_guard<std::mutex> lk(mu_);
  timing_ = on;
}

size_t Executor::take_timings(float* ms, size_t cap) {
  std::lock_guard<std::mutex> lk(mu_);
  DeviceGuard g(device_);
  size_t n = 0;
  for (auto& pr : timed_) {
    GCU(cudaEventSynchronize(pr.second));
    float t = 0.f;
    GCU(cudaEventElapsedTime(&t, pr.first, pr.second));
    if (ms && n < cap) ms[n] = t;
    ++n;
    ev_pool_.push_back(pr.first);
    ev_pool_.push_back(pr.second);
  }
  timed_.clear();
  return n;
}

void Executor::set_yield_every(uint64_t every) {
  std::lock_guard<std::mutex> lk(mu_);
  hctrl_->yield_every = every;
}

void Executor::set_debug_level(int level) {
  std::lock_guard<std::mutex> lk(mu_);
  debug_level_ = level;
  hctrl_->debug_level = (uint32_t)level;
}

void Executor::stall_next_batch() {
  std::lock_guard<std::mutex> lk(mu_);
  stall_next_ = true;
}

void Executor::stats(gpuos_stats* out) {
  std::lock_guard<std::mutex> lk(mu_);
  reclaim();
  std::memset(out, 0, sizeof(*out));
  out->published = next_seq_;
  out->staged = opt_.mode == GPUOS_MODE_PERSISTENT ? hctrl_->staged : next_seq_;
  out->processed = done_wm_;
  out->retired = retired_wm_;
  out->heartbeat = hctrl_->heartbeat;
  out->requests = requests_;
  out->pending = pending_.size();
  out->errors = errors_;
  out->relaunches = relaunches_;
  out->dev_ns = dev_ns_;
  out->lean = lean_count_;
  out->chain = chain_count_;
  out->capacity = opt_.capacity;
  out->max_batch = opt_.max_batch;
  out->mode = opt_.mode;
  out->worker_alive = 0;
  if (opt_.mode == GPUOS_MODE_PERSISTENT && worker_launched_) {
    DeviceGuard g(device_);
    out->worker_alive = cudaStreamQuery(s_worker_) == cudaErrorNotReady ? 1 : 0;
  }
  out->quit = (int32_t)hctrl_->quit;
  out->grid = opt_.mode == GPUOS_MODE_PERSISTENT ? grid_ : sm_count_ * batch_bps_;
  out->block = block_;
  out->device = device_;
}

void Executor::shutdown() {
  {
    std::lock_guard<std::mutex> lk(mu_);
    if (!started_) return;
  }
  std::string first_error;
  try {
    flush(true, nullptr);
  } catch (const std::exception& e) {
    first_error = e.what();
  }
  std::lock_guard<std::mutex> lk(mu_);
  DeviceGuard g(device_);
  started_ = false;
  if (worker_launched_) {
    hctrl_->quit = 1u;
    std::atomic_thread_fence(std::memory_order_seq_cst);
    const auto t0 = std::chrono::steady_clock::now();
    bool stopped = true;
    while (cudaStreamQuery(s_worker_) == cudaErrorNotReady) {
      const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
      if (el > sync_timeout_s_ + idle_ns_ * 1e-9) {
        stopped = false;
        break;
      }
      std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    worker_launched_ = false;
    if (!stopped) {
      // Freeing device memory synchronises the device, which would wait for
      // the worker without bound: leave the executor's memory to process exit.
      throw GError(GPUOS_ETIMEOUT,
                   "the persistent worker did not stop (exit reason " +
                       std::to_string(hctrl_->exit_reason) + ", worker errors " +
                       std::to_string(hctrl_->err) + ", staged " +
                       std::to_string(hctrl_->staged) + ", processed " +
                       std::to_string(hctrl_->processed) + ", published " +
                       std::to_string(next_seq_) + "); its memory is left allocated" +
                       (first_error.empty() ? std::string() : "; " + first_error));
    }
  }
  cudaStreamSynchronize(s_own_);
  cudaStreamSynchronize(s_ctrl_);
  if (s_copy_) cudaStreamSynchronize(s_copy_);
  if (states_) cudaFree(states_);
  for (JitKernel& k : jit_kernels_) jit_unload(k);
  jit_kernels_.clear();
  if (jit_state_) cudaFree(jit_state_);
  if (jit_word_) cudaFreeHost(const_cast<uint64_t*>(jit_word_));
  jit_state_ = nullptr;
  jit_word_ = nullptr;
  if (ring_) cudaFree(ring_);
  if (dctrl_) cudaFree(dctrl_);
  if (dtab_) cudaFree(dtab_);
  for (cudaEvent_t& e : done_ev_)
    if (e) cudaEventDestroy(e);
  for (cudaEvent_t& e : copy_ev_)
    if (e) cudaEventDestroy(e);
  if (partials_) cudaFree(partials_);
  if (counters_) cudaFree(counters_);
  if (arena_) cudaFreeHost(arena_);
  if (hostblk_) cudaFreeHost(hostblk_);
  if (last_event_) cudaEventDestroy(last_event_);
  for (auto& pr : timed_) {
    cudaEventDestroy(pr.first);
    cudaEventDestroy(pr.second);
  }
  for (cudaEvent_t e : ev_pool_) cudaEventDestroy(e);
  timed_.clear();
  ev_pool_.clear();
  if (s_worker_) cudaStreamDestroy(s_worker_);
  if (s_ctrl_) cudaStreamDestroy(s_ctrl_);
  if (s_own_) cudaStreamDestroy(s_own_);
  if (s_copy_) cudaStreamDestroy(s_copy_);
  s_copy_ = nullptr;
  states_ = nullptr; ring_ = nullptr; dctrl_ = nullptr; dtab_ = nullptr; partials_ = nullptr; counters_ = nullptr;
  arena_ = nullptr; hostblk_ = nullptr; last_event_ = nullptr;
  s_worker_ = s_ctrl_ = s_own_ = nullptr;
  if (!first_error.empty()) throw GError(GPUOS_EDEVICE, "shutdown: " + first_error);
}

}  // namespace gpuos

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
using gpuos::Executor;
using gpuos::GError;

namespace gpuos {
// Lets the other translation units of this library report a message through
// gpuos_last_error().
void set_last_error(const char* msg) { t_last_error = msg; }
}  // namespace gpuos

namespace {
template <class F>
int32_t guard(F&& f) {
  try {
    f();
    return GPUOS_OK;
  } catch (const GError& e) {
    gpuos::t_last_error = e.what();
    return e.code;
  } catch (const std::exception& e) {
    gpuos::t_last_error = e.what();
    return GPUOS_EINVAL;
  } catch (...) {
    gpuos::t_last_error = "unknown error";
    return GPUOS_EINVAL;
  }
}
Executor* X(gpuos_executor* ex) {
  if (!ex) throw GError(GPUOS_ESTATE, "executor handle is NULL");
  return reinterpret_cast<Executor*>(ex);
}
}  // namespace

extern "C" {

int32_t gpuos_abi_version(void) { return GPUOS_ABI_VERSION; }

const char* gpuos_last_error(void) { return gpuos::t_last_error.c_str(); }

// The executor most recently created on each device (the reference-named
// hot-swap shims act on it).
namespace {
std::mutex g_cur_mu;
Executor* g_cur[64] = {nullptr};
}  // namespace

int32_t gpuos_executor_create(int32_t device, const gpuos_options* opt, gpuos_executor** out) {
  return guard([&] {
    if (!out) throw GError(GPUOS_EINVAL, "out is NULL");
    gpuos_options o;
    std::memset(&o, 0, sizeof(o));
    if (opt) o = *opt;
    Executor* e = new Executor(device, o);
    *out = reinterpret_cast<gpuos_executor*>(e);
    std::lock_guard<std::mutex> lk(g_cur_mu);
    if (device >= 0 && device < 64) g_cur[device] = e;
  });
}

int32_t gpuos_executor_destroy(gpuos_executor* ex) {
  return guard([&] {
    Executor* e = X(ex);
    {
      std::lock_guard<std::mutex> lk(g_cur_mu);
      for (Executor*& c : g_cur)
        if (c == e) c = nullptr;
    }
    std::unique_ptr<Executor> hold(e);
    e->shutdown();
  });
}

// cudaSuccess / cudaErrorInvalidValue, as the reference's shims return
static int32_t shim(const std::function<void(Executor*)>& f) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    gpuos::set_last_error("no current CUDA device");
    return 1;
  }
  std::lock_guard<std::mutex> lk(g_cur_mu);
  if (!g_cur[dev]) {
    gpuos::set_last_error("no executor was created on the current device");
    return 1;
  }
  const int32_t rc = guard([&] { f(g_cur[dev]); });
  return rc == GPUOS_OK ? 0 : 1;
}

int32_t gpu_set_op_table_async(int32_t index, uint64_t fn, void* stream) {
  (void)stream;
  return shim([&](Executor* e) { e->set_slot(index, (int)(int64_t)fn, 0.f, 0.f); });
}

int32_t gpu_set_alias_async(int32_t logical_id, int32_t physical_slot, void* stream) {
  (void)stream;
  return shim([&](Executor* e) { e->set_alias(logical_id, physical_slot); });
}

int32_t gpuos_submit_builtin(gpuos_executor* ex, int32_t op, const gpuos_tensor* a,
                             const gpuos_tensor* b, const gpuos_tensor* out) {
  return guard([&] {
    if (op < 0 || op > 3) throw GError(GPUOS_EINVAL, "builtin op must be 0..3 (add, mul, sub, div)");
    if (!a || !b || !out) throw GError(GPUOS_EINVAL, "a, b and out are required");
    X(ex)->submit_ew(op, false, 0.f, 0.f, a, b, *out);
  });
}

int32_t gpuos_submit_unary(gpuos_executor* ex, int32_t slot, const gpuos_tensor* a,
                           const gpuos_tensor* out) {
  return guard([&] {
    if (!a || !out) throw GError(GPUOS_EINVAL, "a and out are required");
    if (slot < 0 || slot >= gpuos::kMaxSlots) throw GError(GPUOS_EINVAL, "slot out of range");
    X(ex)->submit_ew(slot, true, 0.f, 0.f, a, nullptr, *out);
  });
}

int32_t gpuos_submit_binary(gpuos_executor* ex, int32_t slot, const gpuos_tensor* a,
                            const gpuos_tensor* b, const gpuos_tensor* out) {
  return guard([&] {
    if (!a || !b || !out) throw GError(GPUOS_EINVAL, "a, b and out are required");
    if (slot < 0 || slot >= gpuos::kMaxSlots) throw GError(GPUOS_EINVAL, "slot out of range");
    X(ex)->submit_ew(slot, true, 0.f, 0.f, a, b, *out);
  });
}

int32_t gpuos_submit_nary(gpuos_executor* ex, int32_t slot, int32_t nin,
                          const gpuos_tensor* ins, const gpuos_tensor* out) {
  return guard([&] {
    if (!ins || !out) throw GError(GPUOS_EINVAL, "inputs and out are required");
    if (nin < 1 || nin > 4) throw GError(GPUOS_EINVAL, "a request takes 1 to 4 inputs");
    if (nin <= 2) {
      X(ex)->submit_ew(slot, true, 0.f, 0.f, &ins[0], nin == 2 ? &ins[1] : nullptr, *out);
      return;
    }
    const gpuos_tensor* p[4] = {&ins[0], &ins[1], &ins[2], nin > 3 ? &ins[3] : nullptr};
    X(ex)->submit_nary(slot, p, nin, *out);
  });
}
int32_t gpuos_register_elementwise(gpuos_executor* ex, const char* key, const char* expr,
                                   int32_t arity, int32_t* slot_out) {
  return guard([&] {
    if (!key || !expr || !slot_out) throw GError(GPUOS_EINVAL, "key, expr and slot_out are required");
    *slot_out = X(ex)->register_elementwise(key, expr, arity);
  });
}

int32_t gpuos_register_reduce(gpuos_executor* ex, const char* key, const char* op_name,
                              int32_t* slot_out) {
  return guard([&] {
    if (!key || !op_name || !slot_out) throw GError(GPUOS_EINVAL, "key, op_name and slot_out are required");
    *slot_out = X(ex)->register_reduce(key, op_name);
  });
}

int32_t gpuos_submit_reduce(gpuos_executor* ex, int32_t slot, const gpuos_tensor* x,
                            const gpuos_tensor* out, const int32_t* axes, int32_t naxes,
                            int32_t keepdim) {
  return guard([&] {
    if (!x || !out) throw GError(GPUOS_EINVAL, "x and out are required");
    if (naxes < 0 || naxes > 8 || (naxes > 0 && !axes)) throw GError(GPUOS_EINVAL, "bad axes");
    if (slot < 0 || slot >= gpuos::kMaxSlots) throw GError(GPUOS_EINVAL, "slot out of range");
    X(ex)->submit_reduce(slot, true, *x, *out, axes, naxes, keepdim != 0);
  });
}

int32_t gpuos_submit_task(gpuos_executor* ex, const void* task) {
  return guard([&] {
    if (!task) throw GError(GPUOS_EINVAL, "task is NULL");
    X(ex)->submit_task(task);
  });
}

int32_t gpuos_flush(gpuos_executor* ex, int32_t sync, void* stream, uint64_t* ticket_out) {
  return guard([&] {
    const uint64_t t = X(ex)->flush(sync != 0, static_cast<cudaStream_t>(stream));
    if (ticket_out) *ticket_out = t;
  });
}

int32_t gpuos_wait(gpuos_executor* ex, uint64_t ticket, double timeout_s) {
  return guard([&] { X(ex)->wait(ticket, timeout_s); });
}

int32_t gpuos_set_alias(gpuos_executor* ex, int32_t logical, int32_t physical) {
  return guard([&] { X(ex)->set_alias(logical, physical); });
}

int32_t gpuos_set_slot(gpuos_executor* ex, int32_t slot, int32_t variant, float p0, float p1) {
  return guard([&] { X(ex)->set_slot(slot, variant, p0, p1); });
}

int32_t gpuos_get_slot(gpuos_executor* ex, int32_t slot, int32_t* variant, float* p0, float* p1,
                       int32_t* alias) {
  return guard([&] {
    int v = 0, al = 0;
    X(ex)->get_slot(slot, &v, p0, p1, &al);
    if (variant) *variant = v;
    if (alias) *alias = al;
  });
}

int32_t gpuos_variant_by_name(const char* name) {
  return name ? gpuos::variant_by_name(name) : -1;
}

int32_t gpuos_set_timing(gpuos_executor* ex, int32_t on) {
  return guard([&] { X(ex)->set_timing(on != 0); });
}

int32_t gpuos_take_timings(gpuos_executor* ex, float* ms, uint64_t cap, uint64_t* n_out) {
  return guard([&] {
    const size_t n = X(ex)->take_timings(ms, (size_t)cap);
    if (n_out) *n_out = n;
  });
}

int32_t gpuos_set_yield_every(gpuos_executor* ex, uint64_t every) {
  return guard([&] { X(ex)->set_yield_every(every); });
}

int32_t gpuos_set_debug_level(gpuos_executor* ex, int32_t level) {
  return guard([&] { X(ex)->set_debug_level(level); });
}

int32_t gpuos_debug_stall_next_batch(gpuos_executor* ex) {
  return guard([&] { X(ex)->stall_next_batch(); });
}

int32_t gpuos_worker_alive(gpuos_executor* ex) {
  int32_t alive = 0;
  int32_t rc = guard([&] { alive = X(ex)->worker_alive() ? 1 : 0; });
  return rc < 0 ? rc : alive;
}

int32_t gpuos_plan_elementwise(int32_t variant, float p0, float p1, const gpuos_tensor* a,
                               const gpuos_tensor* b, const gpuos_tensor* out, gpuos_plan* plan) {
  return guard([&] {
    if (!a || !out || !plan) throw GError(GPUOS_EINVAL, "a, out and plan are required");
    gpuos::Pending p;
    gpuos::build_ew(p, variant, false, p0, p1, a, b, *out);
    std::memcpy(plan->record, &p.r, sizeof(p.r));
    plan->nchunk = p.nchunk;
    plan->has_ext = p.has_ext ? 1u : 0u;
    plan->partials = p.partials;
    plan->counters = p.counters;
  });
}

int32_t gpuos_plan_reduce(int32_t variant, const gpuos_tensor* x, const gpuos_tensor* out,
                          const int32_t* axes, int32_t naxes, int32_t keepdim, gpuos_plan* plan) {
  return guard([&] {
    if (!x || !out || !plan) throw GError(GPUOS_EINVAL, "x, out and plan are required");
    if (naxes < 0 || naxes > 8 || (naxes > 0 && !axes)) throw GError(GPUOS_EINVAL, "bad axes");
    gpuos::Pending p;
    gpuos::build_reduce(p, variant, false, *x, *out, axes, naxes, keepdim != 0);
    std::memcpy(plan->record, &p.r, sizeof(p.r));
    plan->nchunk = p.nchunk;
    plan->has_ext = p.has_ext ? 1u : 0u;
    plan->partials = p.partials;
    plan->counters = p.counters;
  });
}

int32_t gpuos_match_expression(const char* expr, int32_t arity, int32_t* variant, float* p0,
                               float* p1) {
  return guard([&] {
    if (!expr || !variant) throw GError(GPUOS_EINVAL, "expr and variant are required");
    float a = 0.f, b = 0.f;
    *variant = gpuos::match_builtin_expr(expr, arity, &a, &b);
    if (p0) *p0 = a;
    if (p1) *p1 = b;
  });
}

int32_t gpuos_get_stats(gpuos_executor* ex, gpuos_stats* out) {
  return guard([&] {
    if (!out) throw GError(GPUOS_EINVAL, "out is NULL");
    X(ex)->stats(out);
  });
}

}  // extern "C"

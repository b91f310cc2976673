// Multi-process sharing: several client processes feed one per-GPU executor.
//
// The reference runs one persistent kernel per process and leaves the
// sharing of a GPU between processes to MPS (benchmarks/bench_mps.py:54-92:
// every worker process calls gpuos_ext.init, submit_add and flush on its own).
// Here one server owns the GPU's executor and a device memory pool that it
// exports with CUDA IPC; each client process maps the pool, places its
// tensors in its own region of it, and writes its requests into its own
// single-producer ring in POSIX shared memory.  The server thread drains
// every client's ring into the one executor, so requests from different
// processes share batches (one launch for all the clients that flushed in
// the same round), and posts each client's completion back into the shared
// memory.
//
// Shared memory "/<name>": Header | ClientCtl[max_clients] |
// Entry[max_clients][ring_entries].  An Entry carries gpuos_tensor
// descriptors whose `data` field is a byte offset into the pool.  Every
// counter is monotonic: a client that takes over a freed slot continues from
// its tail.
//
// Record mode (device < 0): no GPU, no pool and no executor; the server counts
// what it receives and completes every flush at once.  It exercises the
// protocol (rings, flush markers, mailbox, dead clients) on machines without
// a GPU.
#include <cuda_runtime.h>
#include <errno.h>
#include <fcntl.h>
#include <signal.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "runtime.h"

namespace gpuos {
void set_last_error(const char* msg);
}

namespace {

using namespace gpuos;

constexpr uint32_t kMagic = 0x49534f47u;  // "GOSI"
constexpr uint32_t kVersion = 1;
constexpr int kMaxIn = 4;

enum EntryType : uint32_t { IE_BUILTIN = 1, IE_SLOT = 2, IE_REDUCE = 3, IE_FLUSH = 4 };
enum MailKind : int32_t { MB_ELEMENTWISE = 1, MB_REDUCE = 2 };

struct alignas(64) Entry {
  uint32_t type;
  int32_t op;        // IE_BUILTIN: GPUOS_OP_*; IE_SLOT / IE_REDUCE: jump-table slot
  int32_t nin;       // inputs t[0..nin-1]; t[nin] is the output
  int32_t naxes;     // IE_REDUCE
  int32_t keepdim;
  int32_t sync;      // IE_FLUSH: the client waits for it
  int32_t axes[8];
  gpuos_tensor t[kMaxIn + 1];
};

struct alignas(64) ClientCtl {
  uint64_t tail;        // client: entries written
  uint64_t pad0[7];
  uint64_t head;        // server: entries taken
  uint64_t done;        // server: entries complete (up to the last completed flush)
  int32_t status;       // server: first error since the client last read it
  int32_t pad1;
  uint64_t pad2[5];
  int32_t pid;          // owner, 0 = free
  int32_t pad3;
  uint64_t region_off;  // the client's region of the pool
  uint64_t region_bytes;
  uint64_t pad4[5];
  uint64_t mb_req;      // client: registration request number
  uint64_t mb_resp;     // server: answered request number
  int32_t mb_kind, mb_arity, mb_result, mb_rc;
  char mb_key[256];
  char mb_expr[2048];
  char mb_err[256];
  char err[256];        // message of `status`
};

struct alignas(64) Header {
  uint32_t magic, version;
  int32_t device;       // < 0: record mode
  int32_t max_clients;
  uint32_t ring_entries;
  int32_t server_pid;
  uint64_t pool_bytes;
  uint64_t fake_base;   // record mode: the pool address range clients use
  uint64_t heartbeat;   // server loop rounds
  uint32_t alive;       // 1 while the server runs
  uint32_t pad;
  uint8_t handle[64];   // cudaIpcMemHandle_t of the pool
  uint64_t requests;    // requests taken
  uint64_t client_flushes;
  uint64_t launch_flushes;  // executor flushes (one per round with flush markers)
};
static_assert(sizeof(cudaIpcMemHandle_t) <= 64, "IPC handle size");

template <class T>
T ld_acq(const T* p) { return __atomic_load_n(p, __ATOMIC_ACQUIRE); }
template <class T>
void st_rel(T* p, T v) { __atomic_store_n(p, v, __ATOMIC_RELEASE); }

size_t layout_bytes(int max_clients, uint32_t ring) {
  return sizeof(Header) + sizeof(ClientCtl) * (size_t)max_clients +
         sizeof(Entry) * (size_t)max_clients * ring;
}

int esize(int dt) { return dt == kF32 ? 4 : 2; }

// Byte range [lo, hi) relative to `data` that a descriptor covers.
bool span_of(const gpuos_tensor& t, int64_t* lo, int64_t* hi) {
  if (t.ndim < 0 || t.ndim > 8) return false;
  int64_t l = 0, h = 0;
  for (int d = 0; d < t.ndim; ++d) {
    if (t.sizes[d] < 0) return false;
    if (t.sizes[d] == 0) {
      *lo = *hi = 0;
      return true;
    }
    const int64_t s = t.strides[d] * (t.sizes[d] - 1);
    if (s < 0) l += s; else h += s;
  }
  const int e = esize(t.dtype);
  *lo = l * e;
  *hi = (h + 1) * e;
  return true;
}

std::string shm_path(const char* name) {
  std::string n = name ? name : "";
  if (n.empty() || n.size() > 200 || n.find('/') != std::string::npos)
    throw GError(GPUOS_EINVAL, "IPC name must be 1 to 200 characters without '/'");
  return "/" + n;
}

void backoff(int it) {
  if (it < 64) std::this_thread::yield();
  else std::this_thread::sleep_for(std::chrono::microseconds(it < 1024 ? 5 : 50));
}

}  // namespace

// ---------------------------------------------------------------------------
// server
// ---------------------------------------------------------------------------
struct gpuos_ipc_server {
  std::string path;
  int fd = -1;
  void* map = nullptr;
  size_t map_bytes = 0;
  Header* h = nullptr;
  ClientCtl* cl = nullptr;
  Entry* ring = nullptr;
  gpuos::Executor* ex = nullptr;
  uint8_t* pool = nullptr;
  std::thread th;
  std::atomic<bool> stop{false};
  std::atomic<int> clients{0};
  int rec_slots = 0;  // record mode: the next registration's slot

  struct Pend {
    int c;
    uint64_t pos;
    uint64_t ticket;
  };
  std::vector<Pend> pend;

  void fail(ClientCtl& k, int code, const std::string& msg) {
    if (k.status == 0) {
      std::snprintf(k.err, sizeof(k.err), "%s", msg.c_str());
      st_rel(&k.status, code);
    }
  }

  // descriptor with a pool offset -> descriptor with a device pointer
  bool translate(ClientCtl& k, gpuos_tensor& t) {
    int64_t lo = 0, hi = 0;
    const uint64_t off = reinterpret_cast<uint64_t>(t.data);
    if (!span_of(t, &lo, &hi) || (int64_t)off + lo < 0 || off + (uint64_t)hi > h->pool_bytes ||
        (t.dtype != kF32 && t.dtype != kF16 && t.dtype != kBF16)) {
      fail(k, GPUOS_EINVAL, "a tensor lies outside the shared pool or has a bad descriptor");
      return false;
    }
    t.data = (h->device >= 0 ? pool : nullptr) + off;
    return true;
  }

  void submit(ClientCtl& k, const Entry& e0) {
    Entry e = e0;
    if (e.nin < 1 || e.nin > kMaxIn) {
      fail(k, GPUOS_EINVAL, "bad entry");
      return;
    }
    for (int i = 0; i <= e.nin; ++i)
      if (!translate(k, e.t[i])) return;
    h->requests += 1;
    if (!ex) return;  // record mode
    try {
      const gpuos_tensor& out = e.t[e.nin];
      switch (e.type) {
        case IE_BUILTIN:
          ex->submit_ew(e.op, false, 0.f, 0.f, &e.t[0], e.nin > 1 ? &e.t[1] : nullptr, out);
          break;
        case IE_SLOT:
          if (e.nin <= 2) {
            ex->submit_ew(e.op, true, 0.f, 0.f, &e.t[0], e.nin > 1 ? &e.t[1] : nullptr, out);
          } else {
            const gpuos_tensor* p[kMaxIn] = {&e.t[0], &e.t[1], &e.t[2], e.nin > 3 ? &e.t[3] : nullptr};
            ex->submit_nary(e.op, p, e.nin, out);
          }
          break;
        case IE_REDUCE:
          if (e.naxes < 0 || e.naxes > 8) throw GError(GPUOS_EINVAL, "bad reduction axes");
          ex->submit_reduce(e.op, true, e.t[0], out, e.axes, e.naxes, e.keepdim != 0);
          break;
        default:
          throw GError(GPUOS_EINVAL, "bad entry type");
      }
    } catch (const GError& g) {
      fail(k, g.code, g.what());
    } catch (const std::exception& x) {
      fail(k, GPUOS_EINVAL, x.what());
    }
  }

  void mail(ClientCtl& k) {
    k.mb_rc = GPUOS_OK;
    k.mb_err[0] = 0;
    k.mb_key[sizeof(k.mb_key) - 1] = 0;
    k.mb_expr[sizeof(k.mb_expr) - 1] = 0;
    if (!ex) {  // record mode: slots are numbered in order
      k.mb_result = rec_slots++;
      return;
    }
    try {
      if (k.mb_kind == MB_ELEMENTWISE)
        k.mb_result = ex->register_elementwise(k.mb_key, k.mb_expr, k.mb_arity);
      else if (k.mb_kind == MB_REDUCE)
        k.mb_result = ex->register_reduce(k.mb_key, k.mb_expr);
      else
        throw GError(GPUOS_EINVAL, "bad registration kind");
    } catch (const GError& g) {
      k.mb_rc = g.code;
      std::snprintf(k.mb_err, sizeof(k.mb_err), "%s", g.what());
    } catch (const std::exception& x) {
      k.mb_rc = GPUOS_EINVAL;
      std::snprintf(k.mb_err, sizeof(k.mb_err), "%s", x.what());
    }
  }

  void loop() {
    if (h->device >= 0) cudaSetDevice(h->device);
    const int M = h->max_clients;
    const uint32_t N = h->ring_entries;
    int idle = 0;
    auto last_check = std::chrono::steady_clock::now();
    std::vector<std::pair<int, uint64_t>> marks;
    while (!stop.load(std::memory_order_acquire)) {
      bool work = false;
      marks.clear();
      int live = 0;
      for (int c = 0; c < M; ++c) {
        ClientCtl& k = cl[c];
        if (ld_acq(&k.pid) == 0) continue;
        ++live;
        const uint64_t rq = ld_acq(&k.mb_req);
        if (rq != k.mb_resp) {
          mail(k);
          st_rel(&k.mb_resp, rq);
          work = true;
        }
        const uint64_t t = ld_acq(&k.tail);
        uint64_t hd = k.head;
        while (hd < t) {
          const Entry& e = ring[(size_t)c * N + hd % N];
          ++hd;
          if (e.type == IE_FLUSH) {
            marks.emplace_back(c, hd);  // this client's later entries: next round
            break;
          }
          submit(k, e);
        }
        if (hd != k.head) {
          st_rel(&k.head, hd);
          work = true;
        }
      }
      clients.store(live, std::memory_order_relaxed);
      if (!marks.empty()) {
        // one executor flush for every client that flushed in this pass
        h->client_flushes += marks.size();
        h->launch_flushes += 1;
        uint64_t ticket = 0;
        bool ok = true;
        if (ex) {
          try {
            ticket = ex->flush(false, nullptr);
          } catch (const GError& g) {
            ok = false;
            for (auto& m : marks) fail(cl[m.first], g.code, g.what());
          }
        }
        for (auto& m : marks) {
          if (!ex || !ok) st_rel(&cl[m.first].done, m.second);
          else pend.push_back(Pend{m.first, m.second, ticket});
        }
      }
      // completions
      for (size_t i = 0; i < pend.size();) {
        bool fin = false;
        try {
          fin = ex->poll(pend[i].ticket);
        } catch (const GError& g) {
          fin = true;
          // the batch error belongs to the flush that carried it: every client
          // whose requests were in it hears of it
          for (auto& p : pend)
            if (p.ticket <= pend[i].ticket) fail(cl[p.c], g.code, g.what());
        }
        if (fin) {
          st_rel(&cl[pend[i].c].done, pend[i].pos);
          pend[i] = pend.back();
          pend.pop_back();
          work = true;
        } else {
          ++i;
        }
      }
      st_rel(&h->heartbeat, h->heartbeat + 1);
      // clients that exited without disconnecting: free their slots once their
      // rings are drained (requests they wrote run all the same)
      const auto now = std::chrono::steady_clock::now();
      if (now - last_check > std::chrono::milliseconds(50)) {
        last_check = now;
        for (int c = 0; c < M; ++c) {
          ClientCtl& k = cl[c];
          const int pid = ld_acq(&k.pid);
          if (pid == 0 || kill(pid, 0) == 0 || errno != ESRCH) continue;
          bool busy = ld_acq(&k.tail) != k.head;
          for (auto& p : pend) busy = busy || p.c == c;
          if (!busy) {
            int expect = pid;
            __atomic_compare_exchange_n(&k.pid, &expect, 0, false, __ATOMIC_ACQ_REL,
                                        __ATOMIC_ACQUIRE);
          }
        }
      }
      if (work) {
        idle = 0;
      } else {
        backoff(pend.empty() ? idle++ : std::min(idle++, 63));
      }
    }
  }
};

// ---------------------------------------------------------------------------
// client
// ---------------------------------------------------------------------------
struct gpuos_ipc_client {
  int fd = -1;
  void* map = nullptr;
  size_t map_bytes = 0;
  Header* h = nullptr;
  ClientCtl* k = nullptr;
  Entry* ring = nullptr;
  int idx = -1;
  uint8_t* base = nullptr;   // the pool in this process
  bool opened = false;       // base came from cudaIpcOpenMemHandle
  double timeout_s = 60.0;

  void wait_until(const uint64_t* word, uint64_t want, const char* what) {
    const auto t0 = std::chrono::steady_clock::now();
    for (int it = 0; ld_acq(word) < want; ++it) {
      if (!ld_acq(&h->alive)) throw GError(GPUOS_ESTATE, "the IPC server has stopped");
      const double el =
          std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
      if (el > timeout_s) throw GError(GPUOS_ETIMEOUT, std::string("timed out waiting for ") + what);
      backoff(it);
    }
  }

  Entry& next_entry() {
    const uint64_t t = k->tail;
    // room: the server has taken entries up to t - ring_entries
    const uint64_t need = t + 1 > h->ring_entries ? t + 1 - h->ring_entries : 0;
    wait_until(&k->head, need, "room in the IPC ring");
    return ring[(size_t)idx * h->ring_entries + t % h->ring_entries];
  }

  void publish() { st_rel(&k->tail, k->tail + 1); }

  void put_tensor(gpuos_tensor& dst, const gpuos_tensor* src, const char* what) {
    if (!src) throw GError(GPUOS_EINVAL, std::string(what) + " is required");
    dst = *src;
    int64_t lo = 0, hi = 0;
    if (span_of(*src, &lo, &hi) && hi == lo) {  // empty: no memory to locate
      dst.data = nullptr;
      return;
    }
    const uint64_t p = reinterpret_cast<uint64_t>(src->data);
    const uint64_t b = reinterpret_cast<uint64_t>(base);
    if (p < b || p - b >= h->pool_bytes + 1)
      throw GError(GPUOS_EINVAL, std::string(what) + " is not in the shared pool");
    dst.data = reinterpret_cast<void*>(p - b);
  }

  void check_status() {
    const int32_t st = ld_acq(&k->status);
    if (st != 0) {
      const std::string msg = k->err;
      st_rel(&k->status, 0);
      throw GError(st, "IPC server: " + msg);
    }
  }
};

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
namespace {
template <class F>
int32_t ipc_guard(F&& f) {
  try {
    f();
    return GPUOS_OK;
  } catch (const GError& e) {
    set_last_error(e.what());
    return e.code;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return GPUOS_EINVAL;
  }
}
}  // namespace

extern "C" {

int32_t gpuos_ipc_server_create(const char* name, int32_t device, uint64_t pool_bytes,
                                int32_t max_clients, int32_t ring_entries,
                                const gpuos_options* opt, gpuos_ipc_server** out) {
  return ipc_guard([&] {
    if (!out) throw GError(GPUOS_EINVAL, "out is required");
    if (max_clients < 1 || max_clients > 64) throw GError(GPUOS_EINVAL, "max_clients must be 1..64");
    if (ring_entries < 2 || ring_entries > (1 << 16))
      throw GError(GPUOS_EINVAL, "ring_entries must be 2..65536");
    auto* s = new gpuos_ipc_server();
    try {
      s->path = shm_path(name);
      s->map_bytes = layout_bytes(max_clients, (uint32_t)ring_entries);
      s->fd = shm_open(s->path.c_str(), O_RDWR | O_CREAT | O_EXCL, 0600);
      if (s->fd < 0)
        throw GError(GPUOS_EINVAL, "shm_open(" + s->path + "): " + std::strerror(errno));
      if (ftruncate(s->fd, (off_t)s->map_bytes) != 0)
        throw GError(GPUOS_EINVAL, std::string("ftruncate: ") + std::strerror(errno));
      s->map = mmap(nullptr, s->map_bytes, PROT_READ | PROT_WRITE, MAP_SHARED, s->fd, 0);
      if (s->map == MAP_FAILED) {
        s->map = nullptr;
        throw GError(GPUOS_EINVAL, std::string("mmap: ") + std::strerror(errno));
      }
      std::memset(s->map, 0, s->map_bytes);
      s->h = reinterpret_cast<Header*>(s->map);
      s->cl = reinterpret_cast<ClientCtl*>(s->h + 1);
      s->ring = reinterpret_cast<Entry*>(s->cl + max_clients);
      Header& h = *s->h;
      h.device = device;
      h.max_clients = max_clients;
      h.ring_entries = (uint32_t)ring_entries;
      h.server_pid = (int32_t)getpid();
      h.pool_bytes = pool_bytes;
      // each client's region of the pool: an equal share, 2 MB aligned
      const uint64_t share = (pool_bytes / (uint64_t)max_clients) & ~((2ull << 20) - 1);
      for (int c = 0; c < max_clients; ++c) {
        s->cl[c].region_off = share * (uint64_t)c;
        s->cl[c].region_bytes = share;
      }
      if (device >= 0) {
        if (cudaSetDevice(device) != cudaSuccess) throw GError(GPUOS_ECUDA, "cudaSetDevice failed");
        if (pool_bytes == 0) throw GError(GPUOS_EINVAL, "pool_bytes must be positive");
        if (cudaMalloc(reinterpret_cast<void**>(&s->pool), pool_bytes) != cudaSuccess)
          throw GError(GPUOS_ECUDA, "cudaMalloc of the shared pool failed");
        cudaIpcMemHandle_t hd;
        if (cudaIpcGetMemHandle(&hd, s->pool) != cudaSuccess)
          throw GError(GPUOS_ECUDA, "cudaIpcGetMemHandle failed");
        std::memcpy(h.handle, &hd, sizeof(hd));
        gpuos_options o{};
        if (opt) o = *opt;
        else o.mode = GPUOS_MODE_STREAM;
        s->ex = new gpuos::Executor(device, o);
      } else {
        h.fake_base = 1ull << 40;  // record mode: an address range no process maps
      }
      h.version = kVersion;
      st_rel(&h.alive, 1u);
      st_rel(&h.magic, kMagic);
      s->th = std::thread([s] { s->loop(); });
    } catch (...) {
      if (s->ex) delete s->ex;
      if (s->pool) cudaFree(s->pool);
      if (s->map) munmap(s->map, s->map_bytes);
      if (s->fd >= 0) {
        close(s->fd);
        shm_unlink(s->path.c_str());
      }
      delete s;
      throw;
    }
    *out = s;
  });
}

// Stops the server: its thread ends, the executor drains and shuts down, the
// pool is freed and the shared memory name removed.  Clients still connected
// see the server stop (their waits end with GPUOS_ESTATE); their mappings of
// the pool must not be used after this.
int32_t gpuos_ipc_server_destroy(gpuos_ipc_server* s) {
  return ipc_guard([&] {
    if (!s) return;
    s->stop.store(true, std::memory_order_release);
    if (s->th.joinable()) s->th.join();
    int32_t rc = GPUOS_OK;
    std::string msg;
    if (s->ex) {
      try {
        s->ex->flush(true, nullptr);
        s->ex->shutdown();
      } catch (const GError& g) {
        rc = g.code;
        msg = g.what();
      }
      delete s->ex;
    }
    st_rel(&s->h->alive, 0u);
    if (s->pool) cudaFree(s->pool);
    munmap(s->map, s->map_bytes);
    close(s->fd);
    shm_unlink(s->path.c_str());
    delete s;
    if (rc != GPUOS_OK) throw GError(rc, msg);
  });
}

int32_t gpuos_ipc_server_stats(gpuos_ipc_server* s, uint64_t* requests, uint64_t* client_flushes,
                               uint64_t* launch_flushes, int32_t* clients) {
  return ipc_guard([&] {
    if (!s) throw GError(GPUOS_EINVAL, "server is NULL");
    if (requests) *requests = __atomic_load_n(&s->h->requests, __ATOMIC_ACQUIRE);
    if (client_flushes) *client_flushes = __atomic_load_n(&s->h->client_flushes, __ATOMIC_ACQUIRE);
    if (launch_flushes) *launch_flushes = __atomic_load_n(&s->h->launch_flushes, __ATOMIC_ACQUIRE);
    if (clients) *clients = s->clients.load(std::memory_order_relaxed);
  });
}

int32_t gpuos_ipc_connect(const char* name, double timeout_s, gpuos_ipc_client** out) {
  return ipc_guard([&] {
    if (!out) throw GError(GPUOS_EINVAL, "out is required");
    auto* c = new gpuos_ipc_client();
    if (timeout_s > 0) c->timeout_s = timeout_s;
    try {
      const std::string path = shm_path(name);
      c->fd = shm_open(path.c_str(), O_RDWR, 0);
      if (c->fd < 0) throw GError(GPUOS_EINVAL, "no IPC server named " + path);
      struct stat sb;
      if (fstat(c->fd, &sb) != 0 || (size_t)sb.st_size < sizeof(Header))
        throw GError(GPUOS_EINVAL, "the IPC server's shared memory is not ready");
      c->map_bytes = (size_t)sb.st_size;
      c->map = mmap(nullptr, c->map_bytes, PROT_READ | PROT_WRITE, MAP_SHARED, c->fd, 0);
      if (c->map == MAP_FAILED) {
        c->map = nullptr;
        throw GError(GPUOS_EINVAL, std::string("mmap: ") + std::strerror(errno));
      }
      c->h = reinterpret_cast<Header*>(c->map);
      if (ld_acq(&c->h->magic) != kMagic || c->h->version != kVersion)
        throw GError(GPUOS_EINVAL, "not a gpuos IPC server (or another version)");
      if (c->map_bytes < layout_bytes(c->h->max_clients, c->h->ring_entries))
        throw GError(GPUOS_EINVAL, "the IPC server's shared memory is truncated");
      ClientCtl* cl = reinterpret_cast<ClientCtl*>(c->h + 1);
      c->ring = reinterpret_cast<Entry*>(cl + c->h->max_clients);
      const int me = (int)getpid();
      for (int i = 0; i < c->h->max_clients && c->idx < 0; ++i) {
        int expect = 0;
        if (__atomic_compare_exchange_n(&cl[i].pid, &expect, me, false, __ATOMIC_ACQ_REL,
                                        __ATOMIC_ACQUIRE))
          c->idx = i;
      }
      if (c->idx < 0) throw GError(GPUOS_ESTATE, "every client slot of the IPC server is taken");
      c->k = &cl[c->idx];
      st_rel(&c->k->status, 0);
      if (c->h->device >= 0) {
        int prev = 0;
        cudaGetDevice(&prev);
        if (cudaSetDevice(c->h->device) != cudaSuccess)
          throw GError(GPUOS_ECUDA, "cudaSetDevice failed");
        cudaIpcMemHandle_t hd;
        std::memcpy(&hd, c->h->handle, sizeof(hd));
        void* p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, hd, cudaIpcMemLazyEnablePeerAccess);
        cudaSetDevice(prev);
        if (e != cudaSuccess)
          throw GError(GPUOS_ECUDA, std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
        c->base = static_cast<uint8_t*>(p);
        c->opened = true;
      } else {
        c->base = reinterpret_cast<uint8_t*>(c->h->fake_base);
      }
    } catch (...) {
      if (c->k) st_rel(&c->k->pid, 0);
      if (c->map) munmap(c->map, c->map_bytes);
      if (c->fd >= 0) close(c->fd);
      delete c;
      throw;
    }
    *out = c;
  });
}

// Waits for the client's requests, then frees its slot and its mapping.
int32_t gpuos_ipc_disconnect(gpuos_ipc_client* c) {
  return ipc_guard([&] {
    if (!c) return;
    int32_t rc = GPUOS_OK;
    std::string msg;
    try {
      if (ld_acq(&c->h->alive)) {
        const uint64_t t = c->k->tail;
        if (ld_acq(&c->k->done) < t) {
          Entry& e = c->next_entry();
          std::memset(&e, 0, sizeof(Entry));
          e.type = IE_FLUSH;
          e.sync = 1;
          c->publish();
          c->wait_until(&c->k->done, c->k->tail, "the IPC server to finish");
        }
      }
    } catch (const GError& g) {
      rc = g.code;
      msg = g.what();
    }
    if (c->opened && c->h->device >= 0) {
      int prev = 0;
      cudaGetDevice(&prev);
      cudaSetDevice(c->h->device);
      cudaIpcCloseMemHandle(c->base);
      cudaSetDevice(prev);
    }
    st_rel(&c->k->pid, 0);
    munmap(c->map, c->map_bytes);
    close(c->fd);
    delete c;
    if (rc != GPUOS_OK) throw GError(rc, msg);
  });
}

int32_t gpuos_ipc_pool(gpuos_ipc_client* c, void** base, uint64_t* bytes, uint64_t* region_off,
                       uint64_t* region_bytes, int32_t* device) {
  return ipc_guard([&] {
    if (!c) throw GError(GPUOS_EINVAL, "client is NULL");
    if (base) *base = c->base;
    if (bytes) *bytes = c->h->pool_bytes;
    if (region_off) *region_off = c->k->region_off;
    if (region_bytes) *region_bytes = c->k->region_bytes;
    if (device) *device = c->h->device;
  });
}

int32_t gpuos_ipc_submit_builtin(gpuos_ipc_client* c, int32_t op, const gpuos_tensor* a,
                                 const gpuos_tensor* b, const gpuos_tensor* out) {
  return ipc_guard([&] {
    if (!c) throw GError(GPUOS_EINVAL, "client is NULL");
    Entry& e = c->next_entry();
    e.type = IE_BUILTIN;
    e.op = op;
    e.nin = 2;
    c->put_tensor(e.t[0], a, "input A");
    c->put_tensor(e.t[1], b, "input B");
    c->put_tensor(e.t[2], out, "output");
    c->publish();
  });
}

int32_t gpuos_ipc_submit_slot(gpuos_ipc_client* c, int32_t slot, int32_t nin,
                              const gpuos_tensor* ins, const gpuos_tensor* out) {
  return ipc_guard([&] {
    if (!c || !ins) throw GError(GPUOS_EINVAL, "client and inputs are required");
    if (nin < 1 || nin > kMaxIn) throw GError(GPUOS_EINVAL, "a request takes 1 to 4 inputs");
    Entry& e = c->next_entry();
    e.type = IE_SLOT;
    e.op = slot;
    e.nin = nin;
    for (int i = 0; i < nin; ++i) c->put_tensor(e.t[i], &ins[i], "input");
    c->put_tensor(e.t[nin], out, "output");
    c->publish();
  });
}

int32_t gpuos_ipc_submit_reduce(gpuos_ipc_client* c, int32_t slot, const gpuos_tensor* x,
                                const gpuos_tensor* out, const int32_t* axes, int32_t naxes,
                                int32_t keepdim) {
  return ipc_guard([&] {
    if (!c) throw GError(GPUOS_EINVAL, "client is NULL");
    if (naxes < 0 || naxes > 8 || (naxes > 0 && !axes)) throw GError(GPUOS_EINVAL, "bad axes");
    Entry& e = c->next_entry();
    e.type = IE_REDUCE;
    e.op = slot;
    e.nin = 1;
    e.naxes = naxes;
    e.keepdim = keepdim;
    for (int i = 0; i < naxes; ++i) e.axes[i] = axes[i];
    c->put_tensor(e.t[0], x, "input");
    c->put_tensor(e.t[1], out, "output");
    c->publish();
  });
}

// Publish a flush marker; with sync, wait until every request before it is
// complete and raise the first error the server saw for this client.
int32_t gpuos_ipc_flush(gpuos_ipc_client* c, int32_t sync) {
  return ipc_guard([&] {
    if (!c) throw GError(GPUOS_EINVAL, "client is NULL");
    Entry& e = c->next_entry();
    e.type = IE_FLUSH;
    e.sync = sync;
    e.nin = 0;
    c->publish();
    if (sync) c->wait_until(&c->k->done, c->k->tail, "the IPC flush");
    c->check_status();
  });
}

int32_t gpuos_ipc_register(gpuos_ipc_client* c, int32_t kind, const char* key, const char* expr,
                           int32_t arity, int32_t* slot_out) {
  return ipc_guard([&] {
    if (!c || !key || !expr || !slot_out) throw GError(GPUOS_EINVAL, "bad arguments");
    if (kind != MB_ELEMENTWISE && kind != MB_REDUCE) throw GError(GPUOS_EINVAL, "bad kind");
    if (std::strlen(key) >= sizeof(c->k->mb_key) || std::strlen(expr) >= sizeof(c->k->mb_expr))
      throw GError(GPUOS_EINVAL, "key or expression too long for the IPC mailbox");
    ClientCtl& k = *c->k;
    std::snprintf(k.mb_key, sizeof(k.mb_key), "%s", key);
    std::snprintf(k.mb_expr, sizeof(k.mb_expr), "%s", expr);
    k.mb_kind = kind;
    k.mb_arity = arity;
    const uint64_t rq = k.mb_req + 1;
    st_rel(&k.mb_req, rq);
    c->wait_until(&k.mb_resp, rq, "the IPC registration");
    if (k.mb_rc != GPUOS_OK) throw GError(k.mb_rc, std::string("IPC server: ") + k.mb_err);
    *slot_out = k.mb_result;
  });
}

}  // extern "C"

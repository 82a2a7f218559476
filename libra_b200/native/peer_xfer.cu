// peer_xfer: single-box buffer transfer service for the elastic gradient lane
// and peer weight sync.
//
// Role of the reference's ibverbs helper (infra/elastic/native_rdma_verbs_xfer.c:
// device/PD/QP setup :166-227, attribute exchange over TCP :102-120, one SEND of
// the payload with a polled completion and ~30 s timeout :269-332) on a machine
// whose GPUs share an NVSwitch: instead of registering host memory with a NIC,
// the sender exports its buffer (a CUDA IPC handle for device memory, a POSIX
// shared-memory name for host memory) and sends the handle over a control
// socket; the receiving server maps the buffer and copies it into, or adds it
// to, one of its registered destination buffers.  Device-to-device copies and
// reductions run on the receiver's GPU and read the peer memory over NVLink.
//
// Every wait is bounded: socket I/O has send/receive timeouts, and the server
// polls its completion event against the request's deadline, answering
// LPX_ETIMEOUT if the copy has not finished.  The control token is an access
// check for a socket bound to the local box, not cryptographic authentication.
#include <arpa/inet.h>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <fcntl.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/mman.h>
#include <sys/socket.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>

#include "peer_xfer.h"

namespace {

thread_local char g_err[256] = "";

int fail(int code, const char* fmt, const char* a = "", long long b = 0) {
  std::snprintf(g_err, sizeof(g_err), fmt, a, b);
  return code;
}

double now_s() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

constexpr uint32_t kMagic = 0x3158504cu;  // "LPX1"

#pragma pack(push, 1)
struct Request {
  uint32_t magic;
  int32_t op;
  char token[LPX_NAME_LEN];
  char dst_name[LPX_NAME_LEN];
  lpx_handle_t src;
  uint64_t dst_offset;
  uint64_t bytes;
  double timeout_s;
};
struct Response {
  int32_t status;
  char message[160];
};
#pragma pack(pop)

bool send_all(int fd, const void* p, size_t n) {
  const char* c = static_cast<const char*>(p);
  while (n) {
    const ssize_t k = ::send(fd, c, n, MSG_NOSIGNAL);
    if (k <= 0) return false;
    c += k;
    n -= (size_t)k;
  }
  return true;
}

bool recv_all(int fd, void* p, size_t n) {
  char* c = static_cast<char*>(p);
  while (n) {
    const ssize_t k = ::recv(fd, c, n, 0);
    if (k <= 0) return false;
    c += k;
    n -= (size_t)k;
  }
  return true;
}

void set_timeouts(int fd, double seconds) {
  if (seconds <= 0) seconds = 30.0;
  timeval tv;
  tv.tv_sec = (time_t)seconds;
  tv.tv_usec = (suseconds_t)((seconds - (double)tv.tv_sec) * 1e6);
  setsockopt(fd, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof(tv));
  setsockopt(fd, SOL_SOCKET, SO_SNDTIMEO, &tv, sizeof(tv));
}

template <typename T>
__global__ void add_kernel(T* __restrict__ dst, const T* __restrict__ src, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    if constexpr (std::is_same<T, float>::value) {
      dst[i] += src[i];
    } else {
      dst[i] = __float2bfloat16(__bfloat162float(dst[i]) + __bfloat162float(src[i]));
    }
  }
}

struct Buffer {
  void* ptr;
  uint64_t bytes;
  int device;  // -1: host
  int dtype;
};

struct HostMap {
  void* ptr;
  uint64_t bytes;
};

struct Server {
  int fd = -1;
  int port = 0;
  std::string token;
  std::thread thread;
  std::atomic<bool> stop{false};
  std::atomic<long long> served{0};
  std::atomic<long long> failed{0};
  std::mutex mu;
  std::map<std::string, Buffer> buffers;
  std::map<std::string, void*> ipc_maps;     // handle bytes -> mapped device pointer
  std::map<std::string, HostMap> host_maps;  // shm name -> mapping
  std::map<int, cudaStream_t> streams;
  std::map<int, cudaEvent_t> events;
};

int host_map(Server* s, const lpx_handle_t& h, void** out) {
  auto it = s->host_maps.find(h.shm_name);
  if (it != s->host_maps.end() && it->second.bytes >= h.bytes) {
    *out = it->second.ptr;
    return 0;
  }
  const int fd = shm_open(h.shm_name, O_RDONLY, 0);
  if (fd < 0) return fail(LPX_EMAP, "shm_open(%s) failed", h.shm_name);
  void* p = mmap(nullptr, h.bytes, PROT_READ, MAP_SHARED, fd, 0);
  close(fd);
  if (p == MAP_FAILED) return fail(LPX_EMAP, "mmap(%s) failed", h.shm_name);
  if (it != s->host_maps.end()) munmap(it->second.ptr, it->second.bytes);
  s->host_maps[h.shm_name] = HostMap{p, h.bytes};
  *out = p;
  return 0;
}

int device_map(Server* s, const lpx_handle_t& h, void** out) {
  if (h.pid == (int64_t)getpid()) {  // same process: IPC handles cannot be opened here, use the pointer
    *out = reinterpret_cast<void*>(h.local_ptr);
    return 0;
  }
  const std::string key(h.ipc, sizeof(h.ipc));
  auto it = s->ipc_maps.find(key);
  if (it != s->ipc_maps.end()) {
    *out = it->second;
    return 0;
  }
  cudaIpcMemHandle_t mh;
  std::memcpy(&mh, h.ipc, sizeof(mh));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, mh, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(LPX_EMAP, "cudaIpcOpenMemHandle failed: %s", cudaGetErrorString(e));
  s->ipc_maps[key] = p;
  *out = p;
  return 0;
}

int wait_event(cudaEvent_t ev, double deadline) {
  for (;;) {
    const cudaError_t q = cudaEventQuery(ev);
    if (q == cudaSuccess) return 0;
    if (q != cudaErrorNotReady) return fail(LPX_ECUDA, "copy failed: %s", cudaGetErrorString(q));
    if (now_s() > deadline) return fail(LPX_ETIMEOUT, "copy did not finish before the deadline%s", "");
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

int handle_request(Server* s, const Request& r) {
  if (r.magic != kMagic) return fail(LPX_EPROTO, "bad request magic%s", "");
  if (std::strncmp(r.token, s->token.c_str(), LPX_NAME_LEN) != 0) return fail(LPX_EAUTH, "token mismatch%s", "");
  const double deadline = now_s() + (r.timeout_s > 0 ? r.timeout_s : 30.0);
  std::lock_guard<std::mutex> lock(s->mu);
  auto it = s->buffers.find(std::string(r.dst_name, strnlen(r.dst_name, LPX_NAME_LEN)));
  if (it == s->buffers.end()) return fail(LPX_ENOBUF, "unknown destination buffer %s", r.dst_name);
  const Buffer& dst = it->second;
  if (r.dst_offset > dst.bytes || r.bytes > dst.bytes - r.dst_offset || r.src.offset > r.src.bytes ||
      r.bytes > r.src.bytes - r.src.offset)
    return fail(LPX_ERANGE, "transfer of %s%lld bytes is out of range", "", (long long)r.bytes);
  if (r.op != LPX_OP_COPY && r.op != LPX_OP_ADD) return fail(LPX_EPROTO, "unknown op%s", "");
  const size_t esz = dst.dtype == LPX_DTYPE_F32 ? 4 : 2;
  if (r.op == LPX_OP_ADD && (r.bytes % esz || r.dst_offset % esz))
    return fail(LPX_ERANGE, "add needs whole elements%s", "");
  char* dptr = static_cast<char*>(dst.ptr) + r.dst_offset;
  void* base = nullptr;
  int rc = r.src.kind == LPX_KIND_HOST ? host_map(s, r.src, &base) : device_map(s, r.src, &base);
  if (rc) return rc;
  const char* sptr = static_cast<const char*>(base) + r.src.offset;
  if (dst.device < 0) {
    if (r.src.kind != LPX_KIND_HOST) return fail(LPX_EPROTO, "device source into a host destination%s", "");
    if (r.op == LPX_OP_COPY) {
      std::memcpy(dptr, sptr, r.bytes);
    } else if (dst.dtype == LPX_DTYPE_F32) {
      float* d = reinterpret_cast<float*>(dptr);
      const float* x = reinterpret_cast<const float*>(sptr);
      for (size_t i = 0; i < r.bytes / 4; ++i) d[i] += x[i];
    } else {
      return fail(LPX_EPROTO, "host add supports fp32 only%s", "");
    }
    return 0;
  }
  cudaSetDevice(dst.device);
  cudaStream_t& st = s->streams[dst.device];
  cudaEvent_t& ev = s->events[dst.device];
  if (!st && cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess)
    return fail(LPX_ECUDA, "stream creation failed%s", "");
  if (!ev && cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess)
    return fail(LPX_ECUDA, "event creation failed%s", "");
  cudaError_t e = cudaSuccess;
  if (r.op == LPX_OP_COPY) {
    e = cudaMemcpyAsync(dptr, sptr, r.bytes, cudaMemcpyDefault, st);
  } else {
    if (r.src.kind == LPX_KIND_HOST) return fail(LPX_EPROTO, "add from host memory into a device buffer%s", "");
    const size_t n = r.bytes / esz;
    const int threads = 256;
    const int blocks = (int)std::min<size_t>((n + threads - 1) / threads, 148 * 8);
    if (n) {
      if (dst.dtype == LPX_DTYPE_F32)
        add_kernel<float><<<blocks, threads, 0, st>>>(reinterpret_cast<float*>(dptr),
                                                      reinterpret_cast<const float*>(sptr), n);
      else
        add_kernel<__nv_bfloat16><<<blocks, threads, 0, st>>>(reinterpret_cast<__nv_bfloat16*>(dptr),
                                                              reinterpret_cast<const __nv_bfloat16*>(sptr), n);
      e = cudaGetLastError();
    }
  }
  if (e != cudaSuccess) return fail(LPX_ECUDA, "transfer launch failed: %s", cudaGetErrorString(e));
  cudaEventRecord(ev, st);
  return wait_event(ev, deadline);
}

void serve(Server* s) {
  while (!s->stop.load()) {
    pollfd p{s->fd, POLLIN, 0};
    if (poll(&p, 1, 200) <= 0) continue;
    const int c = accept(s->fd, nullptr, nullptr);
    if (c < 0) continue;
    set_timeouts(c, 30.0);
    Request req;
    Response resp{};
    if (recv_all(c, &req, sizeof(req))) {
      set_timeouts(c, req.timeout_s > 0 ? req.timeout_s + 5.0 : 35.0);
      g_err[0] = 0;
      resp.status = handle_request(s, req);
      std::snprintf(resp.message, sizeof(resp.message), "%s", resp.status ? g_err : "ok");
      (resp.status ? s->failed : s->served).fetch_add(1);
      send_all(c, &resp, sizeof(resp));
    }
    close(c);
  }
}

}  // namespace

extern "C" {

const char* lpx_last_error(void) { return g_err; }

int lpx_host_alloc(const char* name, uint64_t bytes, void** out_ptr, lpx_handle_t* out) {
  if (!name || name[0] != '/' || std::strlen(name) >= LPX_NAME_LEN || !bytes || !out_ptr || !out)
    return fail(LPX_EPROTO, "lpx_host_alloc: need a '/name' shorter than 64 bytes and a size%s", "");
  const int fd = shm_open(name, O_CREAT | O_RDWR, 0600);
  if (fd < 0) return fail(LPX_EMAP, "shm_open(%s) failed", name);
  if (ftruncate(fd, (off_t)bytes) != 0) {
    close(fd);
    return fail(LPX_EMAP, "ftruncate(%s) failed", name);
  }
  void* p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (p == MAP_FAILED) return fail(LPX_EMAP, "mmap(%s) failed", name);
  std::memset(out, 0, sizeof(*out));
  out->kind = LPX_KIND_HOST;
  out->device = -1;
  out->bytes = bytes;
  out->pid = (int64_t)getpid();
  out->local_ptr = (uint64_t)(uintptr_t)p;
  std::snprintf(out->shm_name, LPX_NAME_LEN, "%s", name);
  *out_ptr = p;
  return 0;
}

int lpx_host_free(void* ptr, uint64_t bytes, const char* name, int unlink_name) {
  if (ptr) munmap(ptr, bytes);
  if (unlink_name && name) shm_unlink(name);
  return 0;
}

int lpx_export_device(void* dev_ptr, uint64_t bytes, lpx_handle_t* out) {
  if (!dev_ptr || !out) return fail(LPX_EPROTO, "lpx_export_device: null argument%s", "");
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, dev_ptr) != cudaSuccess || attr.type != cudaMemoryTypeDevice)
    return fail(LPX_EPROTO, "lpx_export_device: not a device pointer%s", "");
  // IPC handles name whole allocations: export the allocation base and carry
  // the offset of dev_ptr inside it (caching allocators hand out interior pointers)
  using GetRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static GetRangeFn get_range = nullptr;
  if (!get_range) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn)
      return fail(LPX_ECUDA, "cuMemGetAddressRange is unavailable%s", "");
    get_range = reinterpret_cast<GetRangeFn>(fn);
  }
  CUdeviceptr base = 0;
  size_t range = 0;
  if (get_range(&base, &range, (CUdeviceptr)(uintptr_t)dev_ptr) != CUDA_SUCCESS)
    return fail(LPX_ECUDA, "cuMemGetAddressRange failed%s", "");
  const uint64_t offset = (uint64_t)((uintptr_t)dev_ptr - (uintptr_t)base);
  if (offset + bytes > range) return fail(LPX_ERANGE, "export of %s%lld bytes runs past the allocation", "", (long long)bytes);
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>((uintptr_t)base));
  if (e != cudaSuccess) return fail(LPX_ECUDA, "cudaIpcGetMemHandle failed: %s", cudaGetErrorString(e));
  std::memset(out, 0, sizeof(*out));
  out->kind = LPX_KIND_DEVICE;
  out->device = attr.device;
  out->bytes = offset + bytes;
  out->offset = offset;
  out->pid = (int64_t)getpid();
  out->local_ptr = (uint64_t)(uintptr_t)base;
  std::memcpy(out->ipc, &h, sizeof(h));
  return 0;
}

void* lpx_server_create(const char* host, int port, const char* token) {
  g_err[0] = 0;
  if (!token || std::strlen(token) >= LPX_NAME_LEN) {
    fail(LPX_EPROTO, "lpx_server_create: token must be shorter than 64 bytes%s", "");
    return nullptr;
  }
  const int fd = socket(AF_INET, SOCK_STREAM, 0);
  if (fd < 0) {
    fail(LPX_ECONNECT, "socket() failed%s", "");
    return nullptr;
  }
  int one = 1;
  setsockopt(fd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
  sockaddr_in a{};
  a.sin_family = AF_INET;
  a.sin_port = htons((uint16_t)port);
  if (inet_pton(AF_INET, host && host[0] ? host : "127.0.0.1", &a.sin_addr) != 1 ||
      bind(fd, reinterpret_cast<sockaddr*>(&a), sizeof(a)) != 0 || listen(fd, 64) != 0) {
    close(fd);
    fail(LPX_ECONNECT, "bind/listen on %s failed", host ? host : "");
    return nullptr;
  }
  socklen_t len = sizeof(a);
  getsockname(fd, reinterpret_cast<sockaddr*>(&a), &len);
  Server* s = new Server();
  s->fd = fd;
  s->port = ntohs(a.sin_port);
  s->token = token;
  s->thread = std::thread(serve, s);
  return s;
}

int lpx_server_port(void* srv) { return srv ? static_cast<Server*>(srv)->port : -1; }

int lpx_server_register(void* srv, const char* name, void* ptr, uint64_t bytes, int device, int dtype) {
  if (!srv || !name || !ptr || std::strlen(name) >= LPX_NAME_LEN)
    return fail(LPX_EPROTO, "lpx_server_register: bad argument%s", "");
  if (dtype != LPX_DTYPE_F32 && dtype != LPX_DTYPE_BF16) return fail(LPX_EPROTO, "unknown dtype%s", "");
  Server* s = static_cast<Server*>(srv);
  std::lock_guard<std::mutex> lock(s->mu);
  s->buffers[name] = Buffer{ptr, bytes, device, dtype};
  return 0;
}

int lpx_server_stats(void* srv, long long* served, long long* failed) {
  if (!srv) return LPX_EPROTO;
  Server* s = static_cast<Server*>(srv);
  if (served) *served = s->served.load();
  if (failed) *failed = s->failed.load();
  return 0;
}

int lpx_server_destroy(void* srv) {
  if (!srv) return 0;
  Server* s = static_cast<Server*>(srv);
  s->stop.store(true);
  if (s->thread.joinable()) s->thread.join();
  close(s->fd);
  for (auto& kv : s->ipc_maps) cudaIpcCloseMemHandle(kv.second);
  for (auto& kv : s->host_maps) munmap(kv.second.ptr, kv.second.bytes);
  for (auto& kv : s->events) cudaEventDestroy(kv.second);
  for (auto& kv : s->streams) cudaStreamDestroy(kv.second);
  delete s;
  return 0;
}

int lpx_push(const char* host, int port, const char* token, const char* dst_name, const lpx_handle_t* src,
             uint64_t dst_offset, uint64_t bytes, int op, double timeout_s) {
  g_err[0] = 0;
  if (!src || !dst_name || !token || std::strlen(dst_name) >= LPX_NAME_LEN || std::strlen(token) >= LPX_NAME_LEN)
    return fail(LPX_EPROTO, "lpx_push: bad argument%s", "");
  const int fd = socket(AF_INET, SOCK_STREAM, 0);
  if (fd < 0) return fail(LPX_ECONNECT, "socket() failed%s", "");
  set_timeouts(fd, timeout_s > 0 ? timeout_s + 5.0 : 35.0);
  sockaddr_in a{};
  a.sin_family = AF_INET;
  a.sin_port = htons((uint16_t)port);
  if (inet_pton(AF_INET, host && host[0] ? host : "127.0.0.1", &a.sin_addr) != 1 ||
      connect(fd, reinterpret_cast<sockaddr*>(&a), sizeof(a)) != 0) {
    close(fd);
    return fail(LPX_ECONNECT, "connect to %s failed", host ? host : "");
  }
  Request r;
  std::memset(&r, 0, sizeof(r));
  r.magic = kMagic;
  r.op = op;
  std::snprintf(r.token, LPX_NAME_LEN, "%s", token);
  std::snprintf(r.dst_name, LPX_NAME_LEN, "%s", dst_name);
  r.src = *src;
  r.dst_offset = dst_offset;
  r.bytes = bytes;
  r.timeout_s = timeout_s;
  Response resp{};
  const bool ok = send_all(fd, &r, sizeof(r)) && recv_all(fd, &resp, sizeof(resp));
  close(fd);
  if (!ok) return fail(LPX_ETIMEOUT, "no response from the transfer server%s", "");
  if (resp.status) {
    std::snprintf(g_err, sizeof(g_err), "%s", resp.message);
    return resp.status;
  }
  return 0;
}

}  // extern "C"

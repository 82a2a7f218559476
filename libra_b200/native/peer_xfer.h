// peer_xfer: single-box buffer transfer service (C ABI, loaded with ctypes).
//
// A receiver creates a server, registers destination buffers by name (device
// memory of one of its GPUs, or host memory), and the sender pushes an
// exported source buffer into one of them, as a copy or an element-wise add.
// Source buffers are exported as CUDA IPC handles (device memory; the handle
// names the allocation base and carries the offset) or POSIX shared-memory
// names (host memory from lpx_host_alloc).
#pragma once

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LPX_NAME_LEN 64

enum { LPX_KIND_HOST = 0, LPX_KIND_DEVICE = 1 };
enum { LPX_OP_COPY = 0, LPX_OP_ADD = 1 };
enum { LPX_DTYPE_F32 = 0, LPX_DTYPE_BF16 = 1 };
enum {
  LPX_OK = 0,
  LPX_ECONNECT = 1,  // socket / connect / bind failure
  LPX_EAUTH = 2,     // control token mismatch
  LPX_ENOBUF = 3,    // unknown destination name
  LPX_ERANGE = 4,    // offset/size outside a buffer
  LPX_EMAP = 5,      // cannot map the source (shm or IPC handle)
  LPX_ECUDA = 6,     // CUDA call failed
  LPX_ETIMEOUT = 7,  // no completion / response before the deadline
  LPX_EPROTO = 8     // malformed request or argument
};

typedef struct {
  int32_t kind;
  int32_t device;      // -1 for host memory
  uint64_t bytes;      // bytes addressable from the mapped base
  uint64_t offset;     // start of the exported range inside the mapping
  int64_t pid;         // exporting process
  uint64_t local_ptr;  // base pointer inside the exporting process
  char ipc[64];        // cudaIpcMemHandle_t bytes (device kind)
  char shm_name[LPX_NAME_LEN];  // shared-memory name (host kind)
} lpx_handle_t;

const char* lpx_last_error(void);

int lpx_host_alloc(const char* name, uint64_t bytes, void** out_ptr, lpx_handle_t* out);
int lpx_host_free(void* ptr, uint64_t bytes, const char* name, int unlink_name);
int lpx_export_device(void* dev_ptr, uint64_t bytes, lpx_handle_t* out);

void* lpx_server_create(const char* host, int port, const char* token);
int lpx_server_port(void* srv);
int lpx_server_register(void* srv, const char* name, void* ptr, uint64_t bytes, int device, int dtype);
int lpx_server_stats(void* srv, long long* served, long long* failed);
int lpx_server_destroy(void* srv);

// Blocks until the server answers or timeout_s (+5 s of socket slack) passes.
int lpx_push(const char* host, int port, const char* token, const char* dst_name, const lpx_handle_t* src,
             uint64_t dst_offset, uint64_t bytes, int op, double timeout_s);

#ifdef __cplusplus
}
#endif

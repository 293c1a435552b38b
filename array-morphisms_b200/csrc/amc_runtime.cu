// Runtime of libamcuda: status/error plumbing, host-side fault injection,
// device selection, per-device streams and the buffer registry.
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "amc_internal.h"

namespace amc {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  std::string m = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  g_last_error = m;
  return e == cudaErrorMemoryAllocation ? AMC_ERR_OOM : AMC_ERR_CUDA;
}

bool fault_injected(const char* what) {
  const char* f = getenv("AMC_FAULT");
  if (!f || !*f) return false;
  // comma separated list of operation classes
  std::string s(f);
  size_t pos = 0;
  while (pos <= s.size()) {
    size_t c = s.find(',', pos);
    std::string tok = s.substr(pos, c == std::string::npos ? std::string::npos : c - pos);
    if (tok == what) return true;
    if (c == std::string::npos) break;
    pos = c + 1;
  }
  return false;
}

size_t dtype_size(int32_t d) {
  switch (d) {
    case AMC_F32: case AMC_S32: case AMC_U32: return 4;
    case AMC_F64: case AMC_S64: case AMC_U64: return 8;
  }
  return 0;
}
bool dtype_valid(int32_t d) { return d >= AMC_F32 && d <= AMC_U64; }
bool dtype_float(int32_t d) { return d == AMC_F32 || d == AMC_F64; }

// ------------------------------------------------------------------ registry
static std::mutex g_mu;
static std::unordered_map<uint64_t, Buffer*> g_bufs;
static uint64_t g_next = 1;

uint64_t buf_register(Buffer* b) {
  std::lock_guard<std::mutex> l(g_mu);
  uint64_t h = g_next++;
  g_bufs[h] = b;
  return h;
}

Buffer* buf_get(uint64_t h) {
  std::lock_guard<std::mutex> l(g_mu);
  auto it = g_bufs.find(h);
  return it == g_bufs.end() ? nullptr : it->second;
}

void buf_retain(uint64_t h) {
  Buffer* b = buf_get(h);
  if (b) b->refs.fetch_add(1);
}

void buf_release(uint64_t h) {
  Buffer* b = nullptr;
  {
    std::lock_guard<std::mutex> l(g_mu);
    auto it = g_bufs.find(h);
    if (it == g_bufs.end()) return;
    b = it->second;
    if (b->refs.fetch_sub(1) != 1) return;
    g_bufs.erase(it);
  }
  if (b->owned && b->ptr) {
    int cur = 0;
    cudaGetDevice(&cur);
    if (cur != b->device) cudaSetDevice(b->device);
    cudaFree(b->ptr);
    if (cur != b->device) cudaSetDevice(cur);
  }
  delete b;
}

int buf_alloc(int32_t dtype, int64_t nelem, uint64_t* out) {
  if (!dtype_valid(dtype)) return fail(AMC_ERR_INVALID, "buffer: invalid dtype");
  if (nelem < 0) return fail(AMC_ERR_INVALID, "buffer: negative size");
  if (fault_injected("alloc")) return fail(AMC_ERR_INJECTED, "buffer: injected allocation failure (AMC_FAULT=alloc)");
  Buffer* b = new Buffer();
  b->dtype = dtype;
  b->nelem = nelem;
  cudaGetDevice(&b->device);
  size_t bytes = (size_t)nelem * dtype_size(dtype);
  if (bytes) {
    cudaError_t e = cudaMalloc(&b->ptr, bytes);
    if (e != cudaSuccess) {
      delete b;
      return cuda_fail(e, "cudaMalloc");
    }
  }
  *out = buf_register(b);
  return AMC_OK;
}

// ------------------------------------------------------------------ devices
static std::mutex g_dev_mu;
static std::unordered_map<int, cudaStream_t> g_streams;
static std::unordered_map<int, int> g_sms;

cudaStream_t default_stream() {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> l(g_dev_mu);
  auto it = g_streams.find(dev);
  if (it != g_streams.end()) return it->second;
  // A blocking stream: it orders with the legacy default stream, so work a
  // host enqueued there (uploads, other libraries) completes first.
  cudaStream_t s = nullptr;
  cudaStreamCreateWithFlags(&s, cudaStreamDefault);
  g_streams[dev] = s;
  return s;
}

int num_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> l(g_dev_mu);
  auto it = g_sms.find(dev);
  if (it != g_sms.end()) return it->second;
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (n <= 0) n = 148;
  g_sms[dev] = n;
  return n;
}

int device_check_errors() {
  int rc = fir_check_error();
  if (rc) return rc;
  rc = attention_check_error();
  if (rc) return rc;
  rc = attention_bwd_check_error();
  if (rc) return rc;
  rc = rowpass_check_error();
  if (rc) return rc;
  rc = dist_check_error();
  if (rc) return rc;
  rc = colfold_check_error();
  if (rc) return rc;
  return conv_check_error();
}

}  // namespace amc

using namespace amc;

extern "C" {

int amc_last_error(char* buf, size_t len) {
  if (!buf || !len) return AMC_ERR_INVALID;
  size_t n = g_last_error.size() < len - 1 ? g_last_error.size() : len - 1;
  memcpy(buf, g_last_error.data(), n);
  buf[n] = 0;
  return AMC_OK;
}

int amc_version(int* major, int* minor) {
  if (major) *major = 0;
  if (minor) *minor = 1;
  return AMC_OK;
}

int amc_device_count(int* n) {
  int c = 0;
  cudaError_t e = cudaGetDeviceCount(&c);
  if (e != cudaSuccess) {
    *n = 0;
    return cuda_fail(e, "cudaGetDeviceCount");
  }
  *n = c;
  return AMC_OK;
}

int amc_init(int device) {
  if (fault_injected("init")) return fail(AMC_ERR_INJECTED, "init: injected failure (AMC_FAULT=init)");
  int c = 0;
  AMC_CUDA(cudaGetDeviceCount(&c));
  if (device < 0 || device >= c) return fail(AMC_ERR_INVALID, "amc_init: no such device");
  AMC_CUDA(cudaSetDevice(device));
  cudaDeviceProp p;
  AMC_CUDA(cudaGetDeviceProperties(&p, device));
  if (p.major < 10) return fail(AMC_ERR_UNSUPPORTED, "amc_init: libamcuda is built for sm_100a (B200); device is sm_" +
                                                          std::to_string(p.major) + std::to_string(p.minor));
  default_stream();
  num_sms();
  return AMC_OK;
}

int amc_shutdown(void) {
  std::vector<uint64_t> hs;
  {
    std::lock_guard<std::mutex> l(g_mu);
    for (auto& kv : g_bufs) hs.push_back(kv.first);
  }
  for (uint64_t h : hs) {
    Buffer* b = buf_get(h);
    if (!b) continue;
    b->refs.store(1);
    buf_release(h);
  }
  return AMC_OK;
}

int amc_synchronize(void) {
  AMC_CUDA(cudaStreamSynchronize(default_stream()));
  return device_check_errors();
}

int amc_buf_create(int32_t dtype, int64_t nelem, uint64_t* out) {
  if (!out) return fail(AMC_ERR_INVALID, "amc_buf_create: null out");
  return buf_alloc(dtype, nelem, out);
}

int amc_buf_wrap(void* devptr, int32_t dtype, int64_t nelem, uint64_t* out) {
  if (!out || (!devptr && nelem)) return fail(AMC_ERR_INVALID, "amc_buf_wrap: null pointer");
  if (!dtype_valid(dtype)) return fail(AMC_ERR_INVALID, "amc_buf_wrap: invalid dtype");
  Buffer* b = new Buffer();
  b->ptr = devptr;
  b->dtype = dtype;
  b->nelem = nelem;
  b->owned = false;
  cudaGetDevice(&b->device);
  *out = buf_register(b);
  return AMC_OK;
}

static int check_range(Buffer* b, int64_t bytes, int64_t off) {
  if (!b) return fail(AMC_ERR_INVALID, "unknown buffer handle");
  int64_t cap = b->nelem * (int64_t)dtype_size(b->dtype);
  if (bytes < 0 || off < 0 || off + bytes > cap) return fail(AMC_ERR_INVALID, "buffer copy out of range");
  return AMC_OK;
}

int amc_buf_upload(uint64_t h, const void* host, int64_t bytes, int64_t off) {
  Buffer* b = buf_get(h);
  int rc = check_range(b, bytes, off);
  if (rc) return rc;
  if (!bytes) return AMC_OK;
  cudaStream_t s = default_stream();
  AMC_CUDA(cudaMemcpyAsync((char*)b->ptr + off, host, (size_t)bytes, cudaMemcpyHostToDevice, s));
  AMC_CUDA(cudaStreamSynchronize(s));
  return AMC_OK;
}

int amc_buf_download(uint64_t h, void* host, int64_t bytes, int64_t off) {
  Buffer* b = buf_get(h);
  int rc = check_range(b, bytes, off);
  if (rc) return rc;
  if (!bytes) return AMC_OK;
  cudaStream_t s = default_stream();
  AMC_CUDA(cudaMemcpyAsync(host, (char*)b->ptr + off, (size_t)bytes, cudaMemcpyDeviceToHost, s));
  AMC_CUDA(cudaStreamSynchronize(s));
  return device_check_errors();
}

int amc_buf_upload_async(uint64_t h, const void* host, int64_t bytes, int64_t off, void* stream) {
  Buffer* b = buf_get(h);
  int rc = check_range(b, bytes, off);
  if (rc) return rc;
  if (!bytes) return AMC_OK;
  AMC_CUDA(cudaMemcpyAsync((char*)b->ptr + off, host, (size_t)bytes, cudaMemcpyHostToDevice, pick_stream(stream)));
  return AMC_OK;
}

int amc_buf_download_async(uint64_t h, void* host, int64_t bytes, int64_t off, void* stream) {
  Buffer* b = buf_get(h);
  int rc = check_range(b, bytes, off);
  if (rc) return rc;
  if (!bytes) return AMC_OK;
  AMC_CUDA(cudaMemcpyAsync(host, (char*)b->ptr + off, (size_t)bytes, cudaMemcpyDeviceToHost, pick_stream(stream)));
  return AMC_OK;
}

int amc_buf_copy_async(uint64_t dst, int64_t dst_off, uint64_t src, int64_t src_off, int64_t bytes, void* stream) {
  Buffer* d = buf_get(dst);
  Buffer* s = buf_get(src);
  int rc = check_range(d, bytes, dst_off);
  if (!rc) rc = check_range(s, bytes, src_off);
  if (rc) return rc;
  if (!bytes) return AMC_OK;
  AMC_CUDA(cudaMemcpyAsync((char*)d->ptr + dst_off, (const char*)s->ptr + src_off, (size_t)bytes,
                           cudaMemcpyDeviceToDevice, pick_stream(stream)));
  return AMC_OK;
}

int amc_buf_devptr(uint64_t h, void** out) {
  Buffer* b = buf_get(h);
  if (!b || !out) return fail(AMC_ERR_INVALID, "amc_buf_devptr: unknown buffer");
  *out = b->ptr;
  return AMC_OK;
}

int amc_buf_info(uint64_t h, int32_t* dtype, int64_t* nelem) {
  Buffer* b = buf_get(h);
  if (!b) return fail(AMC_ERR_INVALID, "amc_buf_info: unknown buffer");
  if (dtype) *dtype = b->dtype;
  if (nelem) *nelem = b->nelem;
  return AMC_OK;
}

int amc_buf_free(uint64_t h) {
  if (!buf_get(h)) return fail(AMC_ERR_INVALID, "amc_buf_free: unknown buffer");
  buf_release(h);
  return AMC_OK;
}

}  // extern "C"

// libppyb200: the runtime under every module the b200 backend builds.
//
// It owns, per device: a non-blocking default stream, a scratch arena per stream for
// the temporaries of a call, a status word per stream, and a cache of device buffers
// for calls that arrive with host memory. The reference's device runtime
// (ppy_runtime/cuda.py) binds device 0's primary context and copies every array per
// launch with synchronous copies; here a call's copies and launches are asynchronous on
// one stream and the device buffers are recycled.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/ppyb200.h"

namespace ppyb200 {
int32_t noalloc_prepare(int device);  // noalloc.cu
}  // namespace ppyb200

namespace {

constexpr int kMaxDevices = 64;

struct StreamState {
  void* scratch = nullptr;
  int64_t scratch_bytes = 0;
  int32_t* status = nullptr;   // device word
  int32_t* status_host = nullptr;  // pinned mirror
};

struct DeviceState {
  bool ready = false;
  cudaStream_t stream = nullptr;
  cudaStream_t side = nullptr;         // second stream of host-memory pipelines
  cudaEvent_t forked = nullptr, joined = nullptr;
  int sm_count = 0;
  std::map<void*, StreamState> streams;           // keyed by cudaStream_t
  std::map<int64_t, std::vector<void*>> free_buffers;  // size class -> buffers
  std::map<void*, int64_t> buffer_class;
};

std::mutex g_mutex;
DeviceState g_devices[kMaxDevices];
std::atomic<uint64_t> g_launches{0};
std::atomic<uint64_t> g_allocations{0};  // cudaMalloc calls that succeeded
std::atomic<int32_t> g_pdl{1};            // launches carry the PDL attribute

// cudaMalloc, counted (ppyb200_device_allocations).
cudaError_t counted_malloc(void** pointer, size_t bytes) {
  const cudaError_t error = cudaMalloc(pointer, bytes);
  if (error == cudaSuccess) g_allocations.fetch_add(1);
  return error;
}

thread_local int t_device = -1;
thread_local cudaStream_t t_stream = nullptr;
thread_local bool t_stream_set = false;
thread_local std::string t_error;

int32_t fail(const std::string& message) {
  t_error = message;
  return PPYB200_RAISED;
}

int32_t check(cudaError_t error, const char* what) {
  if (error == cudaSuccess) return PPYB200_OK;
  std::string message = std::string(what) + ": " + cudaGetErrorString(error);
  return fail(message);
}

// The device state of the calling thread, initialised on first use. Caller holds g_mutex.
DeviceState* device_state_locked() {
  if (t_device < 0) {
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return nullptr;
    t_device = device;
  }
  if (t_device >= kMaxDevices) return nullptr;
  DeviceState& state = g_devices[t_device];
  if (!state.ready) {
    if (cudaSetDevice(t_device) != cudaSuccess) return nullptr;
    if (cudaStreamCreateWithFlags(&state.stream, cudaStreamNonBlocking) != cudaSuccess)
      return nullptr;
    cudaDeviceGetAttribute(&state.sm_count, cudaDevAttrMultiProcessorCount, t_device);
    state.ready = true;
  }
  return &state;
}

cudaStream_t current_stream_locked(DeviceState* state) {
  return t_stream_set && t_stream != nullptr ? t_stream : state->stream;
}

StreamState* stream_state_locked(DeviceState* state, cudaStream_t stream) {
  return &state->streams[reinterpret_cast<void*>(stream)];
}

int64_t size_class(int64_t bytes) {
  int64_t c = 256;
  while (c < bytes) c <<= 1;
  return c;
}

}  // namespace

extern "C" {

int32_t ppyb200_abi_version(void) { return PPYB200_ABI_VERSION; }

int32_t ppyb200_device_count(void) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return count;
}

int32_t ppyb200_init(int32_t device) {
  if (device < 0 || device >= kMaxDevices) return fail("ppyb200_init: no such device");
  int32_t status = check(cudaSetDevice(device), "cudaSetDevice");
  if (status != PPYB200_OK) return status;
  t_device = device;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (device_state_locked() == nullptr)
      return fail("ppyb200_init: could not create device state");
  }
  // load the allocation-free reduction's module (its static array) now, while the caller
  // can still afford device memory
  return ppyb200::noalloc_prepare(device);
}

int32_t ppyb200_current_device(void) { return t_device; }

const char* ppyb200_last_error(void) { return t_error.c_str(); }

void ppyb200_set_error(const char* message) { t_error = message ? message : ""; }

int32_t ppyb200_set_stream(void* stream) {
  t_stream = reinterpret_cast<cudaStream_t>(stream);
  t_stream_set = stream != nullptr;
  return PPYB200_OK;
}

void* ppyb200_stream(void) {
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceState* state = device_state_locked();
  if (state == nullptr) return nullptr;
  return reinterpret_cast<void*>(current_stream_locked(state));
}

int32_t ppyb200_sync(void) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(ppyb200_stream());
  return check(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
}

int32_t ppyb200_sm_count(void) {
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceState* state = device_state_locked();
  return state == nullptr ? 0 : state->sm_count;
}

void* ppyb200_scratch(int64_t bytes) {
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceState* state = device_state_locked();
  if (state == nullptr) {
    fail("ppyb200_scratch: no device");
    return nullptr;
  }
  StreamState* ss = stream_state_locked(state, current_stream_locked(state));
  if (bytes <= 0) bytes = 256;
  if (ss->scratch_bytes < bytes) {
    if (ss->scratch != nullptr) {
      // The previous arena may still be read by work queued on this stream.
      cudaStreamSynchronize(current_stream_locked(state));
      cudaFree(ss->scratch);
      ss->scratch = nullptr;
      ss->scratch_bytes = 0;
    }
    int64_t grown = size_class(bytes);
    if (counted_malloc(&ss->scratch, grown) != cudaSuccess) {
      cudaGetLastError();
      fail("ppyb200_scratch: cudaMalloc failed");
      return nullptr;
    }
    ss->scratch_bytes = grown;
  }
  return ss->scratch;
}

int32_t* ppyb200_status_word(void) {
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceState* state = device_state_locked();
  if (state == nullptr) {
    fail("ppyb200_status_word: no device");
    return nullptr;
  }
  cudaStream_t stream = current_stream_locked(state);
  StreamState* ss = stream_state_locked(state, stream);
  if (ss->status == nullptr) {
    if (counted_malloc(reinterpret_cast<void**>(&ss->status), sizeof(int32_t)) != cudaSuccess ||
        cudaMallocHost(&ss->status_host, sizeof(int32_t)) != cudaSuccess) {
      cudaGetLastError();
      fail("ppyb200_status_word: allocation failed");
      return nullptr;
    }
  }
  if (cudaMemsetAsync(ss->status, 0, sizeof(int32_t), stream) != cudaSuccess) {
    fail("ppyb200_status_word: cudaMemsetAsync failed");
    return nullptr;
  }
  return ss->status;
}

int32_t ppyb200_read_status(int32_t* word) {
  int32_t* host = nullptr;
  cudaStream_t stream;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    DeviceState* state = device_state_locked();
    if (state == nullptr) return fail("ppyb200_read_status: no device");
    stream = current_stream_locked(state);
    host = stream_state_locked(state, stream)->status_host;
  }
  if (host == nullptr) return fail("ppyb200_read_status: no status word on this stream");
  int32_t status = check(cudaMemcpyAsync(host, word, sizeof(int32_t), cudaMemcpyDeviceToHost,
                                         stream), "status copy");
  if (status != PPYB200_OK) return status;
  status = check(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
  if (status != PPYB200_OK) return status;
  // Kernels raise 1 (a guard failed: fall back) or 2 (a device function raised, e.g.
  // a loop past its trip bound).
  if (*host >= 2)
    return fail("a device function raised: a loop passed its trip bound or a call failed");
  return *host;
}

void* ppyb200_device_buffer(int64_t bytes) {
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceState* state = device_state_locked();
  if (state == nullptr) {
    fail("ppyb200_device_buffer: no device");
    return nullptr;
  }
  int64_t c = size_class(bytes > 0 ? bytes : 1);
  auto& pool = state->free_buffers[c];
  if (!pool.empty()) {
    void* p = pool.back();
    pool.pop_back();
    return p;
  }
  void* p = nullptr;
  if (counted_malloc(&p, c) != cudaSuccess) {
    cudaGetLastError();
    fail("ppyb200_device_buffer: cudaMalloc failed");
    return nullptr;
  }
  state->buffer_class[p] = c;
  return p;
}

void ppyb200_release_buffer(void* pointer) {
  if (pointer == nullptr) return;
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceState* state = device_state_locked();
  if (state == nullptr) return;
  auto found = state->buffer_class.find(pointer);
  if (found == state->buffer_class.end()) return;
  state->free_buffers[found->second].push_back(pointer);
}

int32_t ppyb200_copy_to_device(void* device_dst, const void* host_src, int64_t bytes) {
  if (bytes <= 0) return PPYB200_OK;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(ppyb200_stream());
  return check(cudaMemcpyAsync(device_dst, host_src, bytes, cudaMemcpyHostToDevice, stream),
               "host-to-device copy");
}

int32_t ppyb200_copy_to_host(void* host_dst, const void* device_src, int64_t bytes) {
  if (bytes <= 0) return PPYB200_OK;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(ppyb200_stream());
  return check(cudaMemcpyAsync(host_dst, device_src, bytes, cudaMemcpyDeviceToHost, stream),
               "device-to-host copy");
}

int32_t ppyb200_copy_rows_to_host(void* host_dst, int64_t host_pitch, const void* device_src,
                                  int64_t device_pitch, int64_t row_bytes, int64_t rows) {
  if (rows <= 0 || row_bytes <= 0) return PPYB200_OK;
  if (host_pitch < row_bytes || device_pitch < row_bytes)
    return fail("ppyb200_copy_rows_to_host: pitches shorter than a row");
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(ppyb200_stream());
  return check(cudaMemcpy2DAsync(host_dst, (size_t)host_pitch, device_src, (size_t)device_pitch,
                                 (size_t)row_bytes, (size_t)rows, cudaMemcpyDeviceToHost, stream),
               "device-to-host row copy");
}

int32_t ppyb200_fork(void** side) {
  if (side == nullptr) return fail("ppyb200_fork: no result pointer");
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceState* state = device_state_locked();
  if (state == nullptr) return fail("ppyb200_fork: no device");
  if (state->side == nullptr) {
    int32_t s = check(cudaStreamCreateWithFlags(&state->side, cudaStreamNonBlocking),
                      "ppyb200_fork: side stream");
    if (s == PPYB200_OK)
      s = check(cudaEventCreateWithFlags(&state->forked, cudaEventDisableTiming), "ppyb200_fork");
    if (s == PPYB200_OK)
      s = check(cudaEventCreateWithFlags(&state->joined, cudaEventDisableTiming), "ppyb200_fork");
    if (s != PPYB200_OK) return s;
  }
  cudaStream_t current = current_stream_locked(state);
  int32_t s = check(cudaEventRecord(state->forked, current), "ppyb200_fork: record");
  if (s == PPYB200_OK)
    s = check(cudaStreamWaitEvent(state->side, state->forked, 0), "ppyb200_fork: wait");
  *side = reinterpret_cast<void*>(state->side);
  return s;
}

int32_t ppyb200_join(void* side) {
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceState* state = device_state_locked();
  if (state == nullptr) return fail("ppyb200_join: no device");
  if (side == nullptr || side != reinterpret_cast<void*>(state->side))
    return fail("ppyb200_join: not this device's side stream");
  int32_t s = check(cudaEventRecord(state->joined, state->side), "ppyb200_join: record");
  if (s == PPYB200_OK)
    s = check(cudaStreamWaitEvent(current_stream_locked(state), state->joined, 0),
              "ppyb200_join: wait");
  return s;
}

int32_t ppyb200_check(int32_t cuda_error, const char* what) {
  return check(static_cast<cudaError_t>(cuda_error), what ? what : "CUDA call");
}

uint64_t ppyb200_launches(void) { return g_launches.load(); }

uint64_t ppyb200_device_allocations(void) { return g_allocations.load(); }

int32_t ppyb200_set_pdl(int32_t enabled) {
  return g_pdl.exchange(enabled != 0 ? 1 : 0);
}

int32_t ppyb200_pdl(void) { return g_pdl.load(std::memory_order_relaxed); }

void ppyb200_count_launches(uint64_t count) { g_launches.fetch_add(count); }

}  // extern "C"

// Host runtime of the CUDA backend (see runtime.h).
#include "runtime.h"

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iterator>
#include <thread>

namespace iec {

// IEEE 754 binary16, round to nearest even (the rounding of
// crates/native-engine/src/half.rs:7-48), written from the format's
// definition.
uint16_t f32_to_half(float v) {
  uint32_t x;
  std::memcpy(&x, &v, 4);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t mant = x & 0x7fffffu;
  const int exp = (int)((x >> 23) & 0xffu);
  if (exp == 0xff) return sign | 0x7c00u | (mant ? 0x200u : 0u);
  const int e = exp - 127 + 15;
  if (e >= 31) return sign | 0x7c00u;
  if (e <= 0) {
    if (e < -10) return sign;
    const uint32_t sig = mant | 0x800000u;
    const uint32_t shift = (uint32_t)(14 - e);
    uint32_t q = sig >> shift;
    const uint32_t rem = sig & ((1u << shift) - 1), halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (q & 1))) q++;
    return sign | (uint16_t)q;
  }
  uint32_t q = ((uint32_t)e << 10) | (mant >> 13);
  const uint32_t rem = mant & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) q++;  // a carry may reach infinity
  return sign | (uint16_t)q;
}

float half_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  uint32_t bits;
  if (e == 0) {
    float mag = (float)m * 5.9604644775390625e-8f;  // m * 2^-24, exact
    return sign ? -mag : mag;
  }
  if (e == 0x1f) bits = sign | 0x7f800000u | (m << 13);
  else bits = sign | ((e + 112) << 23) | (m << 13);
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// -------------------------------------------------------------- weights file
WeightFile WeightFile::read(const std::string& path, const char magic[8]) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw Error(ERR_IO, path + ": cannot open");
  std::vector<uint8_t> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  if (f.bad()) throw Error(ERR_IO, path + ": read failed");
  return parse(bytes.data(), bytes.size(), magic);
}

WeightFile WeightFile::parse(const uint8_t* data, size_t len, const char magic[8]) {
  size_t at = 0;
  auto take = [&](size_t n) -> const uint8_t* {
    if (n > len - at) throw Error(ERR_WEIGHTS, "weights file is truncated");
    const uint8_t* p = data + at;
    at += n;
    return p;
  };
  auto u32 = [&] {
    uint32_t v;
    std::memcpy(&v, take(4), 4);
    return v;
  };
  if (len < 8 || std::memcmp(data, magic, 8) != 0) {
    std::string kind(magic, 8);
    kind = kind.substr(0, kind.find('\0'));
    throw Error(ERR_WEIGHTS, "not a " + kind + " weights file");
  }
  at = 8;
  const uint32_t version = u32();
  if (version != 1)
    throw Error(ERR_WEIGHTS, "weights file version " + std::to_string(version) + ", expected 1");
  const uint32_t count = u32();
  WeightFile wf;
  for (uint32_t i = 0; i < count; i++) {
    uint16_t name_len;
    std::memcpy(&name_len, take(2), 2);
    std::string name(reinterpret_cast<const char*>(take(name_len)), name_len);
    const uint8_t* tr = take(2);
    const uint8_t dtype = tr[0], rank = tr[1];
    if (dtype > 1) throw Error(ERR_WEIGHTS, name + ": unknown type " + std::to_string(dtype));
    const size_t width = dtype == 0 ? 4 : 2;
    HostTensor t;
    t.half = dtype == 1;
    size_t n = 1;
    for (int r = 0; r < rank; r++) {
      const size_t d = u32();
      if (d != 0 && n > SIZE_MAX / d) throw Error(ERR_WEIGHTS, name + ": too large");
      n *= d;
      t.shape.push_back(d);
    }
    if (n > SIZE_MAX / width) throw Error(ERR_WEIGHTS, name + ": too large");
    const uint8_t* p = take(n * width);
    t.values.resize(n);
    if (width == 4) {
      std::memcpy(t.values.data(), p, n * 4);
    } else {
      for (size_t j = 0; j < n; j++) {
        uint16_t h;
        std::memcpy(&h, p + 2 * j, 2);
        t.values[j] = half_to_f32(h);
      }
    }
    if (!wf.tensors_.emplace(name, std::move(t)).second) throw Error(ERR_WEIGHTS, name + ": stored twice");
  }
  if (at != len) throw Error(ERR_WEIGHTS, "trailing bytes after the last tensor");
  return wf;
}

static std::string shape_str(const std::vector<size_t>& s) {
  std::string out = "[";
  for (size_t i = 0; i < s.size(); i++) out += (i ? ", " : "") + std::to_string(s[i]);
  return out + "]";
}

HostTensor WeightFile::take_tensor(const std::string& name, const std::vector<size_t>& shape) {
  auto it = tensors_.find(name);
  if (it == tensors_.end()) throw Error(ERR_WEIGHTS, name + ": missing");
  if (it->second.shape != shape)
    throw Error(ERR_WEIGHTS, name + ": shape " + shape_str(it->second.shape) + ", expected " + shape_str(shape));
  HostTensor t = std::move(it->second);
  tensors_.erase(it);
  return t;
}

void WeightFile::finish() const {
  if (!tensors_.empty()) throw Error(ERR_WEIGHTS, tensors_.begin()->first + ": not used by this model");
}

// ------------------------------------------------------------------ buffers
void DeviceBuffer::reserve(size_t bytes) {
  if (bytes <= bytes_ && ptr_) return;
  release();
  if (bytes == 0) return;
  cudaError_t e = cudaMalloc(&ptr_, bytes);
  if (e != cudaSuccess) {
    ptr_ = nullptr;
    cudaGetLastError();
    throw Error(ERR_GPU, "cudaMalloc of " + std::to_string(bytes) + " bytes: " + cudaGetErrorString(e));
  }
  bytes_ = bytes;
}

void DeviceBuffer::release() {
  if (ptr_) cudaFree(ptr_);
  ptr_ = nullptr;
  bytes_ = 0;
}

void PinnedBuffer::reserve(size_t bytes) {
  if (bytes <= bytes_ && ptr_) return;
  release();
  if (bytes == 0) return;
  cudaError_t e = cudaMallocHost(&ptr_, bytes);
  if (e != cudaSuccess) {
    ptr_ = nullptr;
    cudaGetLastError();
    throw Error(ERR_GPU, "cudaMallocHost of " + std::to_string(bytes) + " bytes: " + cudaGetErrorString(e));
  }
  bytes_ = bytes;
}

void PinnedBuffer::release() {
  if (ptr_) cudaFreeHost(ptr_);
  ptr_ = nullptr;
  bytes_ = 0;
}

// ------------------------------------------------------------------- device
static int env_int(const char* name, int fallback) {
  const char* v = std::getenv(name);
  if (!v || !*v) return fallback;
  char* end = nullptr;
  long x = std::strtol(v, &end, 10);
  return (end && *end == 0) ? (int)x : fallback;
}

int device_count() {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

namespace {
thread_local Device* g_scope_device = nullptr;
}

Device* scoped_device() { return g_scope_device; }

DeviceScope::DeviceScope(Device& d) {
  if (cudaGetDevice(&prev_) != cudaSuccess) {
    cudaGetLastError();
    prev_ = -1;
  }
  d.enter();
  prev_device_ = g_scope_device;
  g_scope_device = &d;
}

DeviceScope::~DeviceScope() {
  g_scope_device = prev_device_;
  if (prev_ >= 0) cudaSetDevice(prev_);
}

Device::Device(const Options& opt) {
  ordinal_ = opt.device >= 0 ? opt.device : env_int("IEC_CUDA_DEVICE", 0);
  timeout_ms_ = opt.timeout_ms > 0 ? opt.timeout_ms : env_int("IEC_TIMEOUT_MS", 120000);
  batch_chunk_ = opt.batch_chunk;
  const int n = device_count();
  if (n == 0) throw Error(ERR_GPU, "no CUDA device");
  if (ordinal_ < 0 || ordinal_ >= n)
    throw Error(ERR_GPU, "CUDA device " + std::to_string(ordinal_) + " of " + std::to_string(n));
  int prev = -1;
  cudaGetDevice(&prev);
  IEC_CUDA(cudaSetDevice(ordinal_));
  cudaDeviceProp prop;
  IEC_CUDA(cudaGetDeviceProperties(&prop, ordinal_));
  if (prop.major != 10 || prop.minor != 0)
    throw Error(ERR_GPU, std::string(prop.name) + ": compute capability " + std::to_string(prop.major) + "." +
                             std::to_string(prop.minor) + ", the kernels are built for sm_100a (B200)");
  name_ = prop.name;
  sms_ = prop.multiProcessorCount;
  IEC_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
  IEC_CUDA(cudaStreamCreateWithFlags(&copy_stream_, cudaStreamNonBlocking));
  dev_err_.reserve(256);
  host_err_.reserve(256);
  IEC_CUDA(cudaMemset(dev_err_.get(), 0, 256));
  IEC_CUDA(cudaDeviceSynchronize());
  if (prev >= 0) cudaSetDevice(prev);
}

Device::~Device() {
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(ordinal_);
  if (!poisoned()) {
    if (stream_) cudaStreamDestroy(stream_);
    if (copy_stream_) cudaStreamDestroy(copy_stream_);
    for (cudaEvent_t e : event_pool_) cudaEventDestroy(e);
  }
  // A poisoned device may still run work; its buffers and streams are leaked
  // rather than freed under it (as the reference's busy flag does).
  if (poisoned()) {
    dev_err_.leak();
    for (auto& e : scratch_) e.second.leak();
  }
  if (prev >= 0) cudaSetDevice(prev);
}

void Device::set_timing(bool on) {
  timing_ = on;
  timed_.clear();
  events_used_ = 0;
}

int Device::time_begin(const std::string& name, double flop, double bytes, cudaStream_t s) {
  if (!timing_) return -1;
  while (event_pool_.size() < events_used_ + 2) {
    cudaEvent_t e;
    IEC_CUDA(cudaEventCreate(&e));
    event_pool_.push_back(e);
  }
  TimedLaunch t;
  t.name = name;
  t.flop = flop;
  t.bytes = bytes;
  t.a = event_pool_[events_used_++];
  t.b = event_pool_[events_used_++];
  IEC_CUDA(cudaEventRecord(t.a, s));
  timed_.push_back(t);
  return (int)timed_.size() - 1;
}

void Device::time_end(int index, cudaStream_t s) {
  if (index >= 0 && (size_t)index < timed_.size()) IEC_CUDA(cudaEventRecord(timed_[index].b, s));
}

float Device::timed_ms(size_t i) {
  if (i >= timed_.size()) return 0.0f;
  wait_event(timed_[i].b);
  float ms = 0.0f;
  IEC_CUDA(cudaEventElapsedTime(&ms, timed_[i].a, timed_[i].b));
  return ms;
}

void Device::enter() {
  if (poisoned()) throw Error(ERR_GPU, "device unusable after an earlier failure: " + poisoned_);
  IEC_CUDA(cudaSetDevice(ordinal_));
}

void Device::wait_event(cudaEvent_t ev) {
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms_);
  int spins = 0;
  while (true) {
    cudaError_t e = cudaEventQuery(ev);
    if (e == cudaSuccess) return;
    if (e != cudaErrorNotReady) {
      std::string msg = std::string("GPU work failed: ") + cudaGetErrorString(e);
      poison(msg);
      throw Error(ERR_GPU, msg);
    }
    if (std::chrono::steady_clock::now() > deadline) {
      std::string msg = "GPU wait timed out after " + std::to_string(timeout_ms_) + " ms";
      poison(msg);
      throw Error(ERR_TIMEOUT, msg);
    }
    if (++spins > 64) std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

void Device::sync(cudaStream_t s) {
  // The kernels' error word comes back with the same wait.
  cudaError_t e = cudaMemcpyAsync(host_err_.get(), dev_err_.get(), sizeof(int), cudaMemcpyDeviceToHost, s);
  cudaEvent_t ev = nullptr;
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventRecord(ev, s);
  if (e != cudaSuccess) {
    if (ev) cudaEventDestroy(ev);
    std::string msg = std::string("queueing a wait: ") + cudaGetErrorString(e);
    poison(msg);
    throw Error(ERR_GPU, msg);
  }
  try {
    wait_event(ev);
  } catch (...) {
    cudaEventDestroy(ev);
    throw;
  }
  cudaEventDestroy(ev);
  check_device_errors();
}

void Device::check_device_errors() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    std::string msg = std::string("CUDA error: ") + cudaGetErrorString(e);
    poison(msg);
    throw Error(ERR_GPU, msg);
  }
  const int err = *host_err_.as<volatile int>();
  if (err != 0) {
    std::string msg = "a kernel's bounded wait ran out (device error word " + std::to_string(err) + ")";
    poison(msg);
    throw Error(ERR_TIMEOUT, msg);
  }
}

// --------------------------------------------------------------- graphs
PassGraph::~PassGraph() { reset(); }

void PassGraph::reset() {
  for (auto& e : entries_)
    if (e.exec) cudaGraphExecDestroy(e.exec);
  entries_.clear();
}

void PassGraph::run(const std::vector<long long>& key, cudaStream_t s,
                    const std::function<void(cudaStream_t)>& body) {
  // Launch timing records events around each launch: such passes run eagerly.
  const Device* d = scoped_device();
  if (!enabled || (d && d->timing())) return body(s);
  Entry* hit = nullptr;
  for (auto& e : entries_)
    if (e.key == key) hit = &e;
  if (!hit) {
    if (entries_.size() == MAX_ENTRIES) {
      auto lru = entries_.begin();
      for (auto it = entries_.begin(); it != entries_.end(); ++it)
        if (it->used < lru->used) lru = it;
      if (lru->exec) cudaGraphExecDestroy(lru->exec);
      entries_.erase(lru);
    }
    entries_.push_back(Entry{key, 0, nullptr, 0});
    hit = &entries_.back();
  }
  hit->used = ++clock_;
  if (hit->exec) {
    IEC_CUDA(cudaGraphLaunch(hit->exec, s));
    return;
  }
  if (hit->seen++ == 0) return body(s);  // the warm run: allocations, attributes
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  IEC_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeRelaxed));
  try {
    body(s);
  } catch (...) {
    cudaStreamEndCapture(s, &graph);
    if (graph) cudaGraphDestroy(graph);
    (void)cudaGetLastError();
    enabled = false;
    throw;
  }
  cudaError_t e = cudaStreamEndCapture(s, &graph);
  if (e == cudaSuccess) e = cudaGraphInstantiate(&exec, graph, 0);
  if (graph) cudaGraphDestroy(graph);
  if (e != cudaSuccess) {
    // Not capturable here: run it the plain way from now on (the captured
    // launches did not execute).
    (void)cudaGetLastError();
    enabled = false;
    return body(s);
  }
  hit->exec = exec;
  IEC_CUDA(cudaGraphLaunch(exec, s));
}

// ------------------------------------------------------------ tensor maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

void encode_tensor_map(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base,
                       const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box) {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    IEC_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !p) throw Error(ERR_GPU, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  cuuint64_t gdim[5], gstride[4];
  cuuint32_t bdim[5], estride[5];
  for (int i = 0; i < rank; i++) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
    if (i + 1 < rank) gstride[i] = strides_bytes[i];
  }
  CUresult r = fn(map, type, (cuuint32_t)rank, const_cast<void*>(base), gdim, gstride, bdim, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw Error(ERR_GPU, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
}

}  // namespace iec

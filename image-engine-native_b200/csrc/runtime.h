// Host runtime of the CUDA backend: errors, the device a model runs on, its
// streams, device and page-locked buffers, bounded waits, TMA descriptors and
// the weights-file reader.
//
// It takes the slot of the reference's Vulkan runtime
// (crates/native-vulkan/src/lib.rs:122-1021: Gpu, Buffer, Steps): one device
// per model, buffers grown on demand with the smaller ones freed first
// (crates/realesrgan-native/src/gpu.rs:132-136), and a failed or timed-out
// wait that poisons the device for every later call (lib.rs:443-480, usable).
// Unlike the reference every wait here is bounded.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <functional>
#include <initializer_list>
#include <map>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace iec {

enum Status { OK = 0, ERR_IO = 1, ERR_WEIGHTS = 2, ERR_INPUT = 3, CANCELLED = 4, ERR_GPU = 5, ERR_TIMEOUT = 6 };

struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define IEC_CUDA(call)                                                                      \
  do {                                                                                      \
    cudaError_t e_ = (call);                                                                \
    if (e_ != cudaSuccess)                                                                  \
      throw ::iec::Error(::iec::ERR_GPU, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

uint16_t f32_to_half(float v);
float half_to_f32(uint16_t h);

// ------------------------------------------------------------- weights file
// crates/native-engine/src/weight_file.rs:28-145: magic, u32 version 1, u32
// count, then per tensor u16 name length, name, u8 type (0 f32 / 1 f16), u8
// rank, u32 dims, values. Every length is checked against what is left of
// the file before it is used; a tensor the model does not take is an error.
struct HostTensor {
  std::vector<size_t> shape;
  bool half = false;
  std::vector<float> values;  // halves widened exactly
};

class WeightFile {
 public:
  static WeightFile read(const std::string& path, const char magic[8]);
  static WeightFile parse(const uint8_t* data, size_t len, const char magic[8]);
  HostTensor take_tensor(const std::string& name, const std::vector<size_t>& shape);
  std::vector<float> take(const std::string& name, const std::vector<size_t>& shape) {
    return take_tensor(name, shape).values;
  }
  void finish() const;

 private:
  std::map<std::string, HostTensor> tensors_;
};

// ------------------------------------------------------------------ device
struct Options {
  int device = -1;
  int timeout_ms = 0;
  int batch_chunk = 0;
};

class DeviceBuffer {
 public:
  DeviceBuffer() = default;
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
  DeviceBuffer(DeviceBuffer&& o) noexcept : ptr_(o.ptr_), bytes_(o.bytes_) {
    o.ptr_ = nullptr;
    o.bytes_ = 0;
  }
  DeviceBuffer& operator=(DeviceBuffer&& o) noexcept {
    if (this != &o) {
      release();
      ptr_ = o.ptr_;
      bytes_ = o.bytes_;
      o.ptr_ = nullptr;
      o.bytes_ = 0;
    }
    return *this;
  }
  // Forget the memory without freeing it (a poisoned device may still use it).
  void leak() {
    ptr_ = nullptr;
    bytes_ = 0;
  }
  ~DeviceBuffer() { release(); }
  // Grow to at least `bytes` (contents not kept); frees the old one first.
  void reserve(size_t bytes);
  void release();
  void* get() const { return ptr_; }
  size_t size() const { return bytes_; }
  template <class T>
  T* as() const { return static_cast<T*>(ptr_); }

 private:
  void* ptr_ = nullptr;
  size_t bytes_ = 0;
};

class PinnedBuffer {
 public:
  PinnedBuffer() = default;
  PinnedBuffer(const PinnedBuffer&) = delete;
  PinnedBuffer& operator=(const PinnedBuffer&) = delete;
  ~PinnedBuffer() { release(); }
  void reserve(size_t bytes);
  void release();
  void* get() const { return ptr_; }
  template <class T>
  T* as() const { return static_cast<T*>(ptr_); }

 private:
  void* ptr_ = nullptr;
  size_t bytes_ = 0;
};

class Device {
 public:
  explicit Device(const Options& opt);
  ~Device();
  Device(const Device&) = delete;
  Device& operator=(const Device&) = delete;

  int ordinal() const { return ordinal_; }
  const std::string& name() const { return name_; }
  int sms() const { return sms_; }
  cudaStream_t stream() const { return stream_; }
  cudaStream_t copy_stream() const { return copy_stream_; }
  int* dev_err() const { return dev_err_.as<int>(); }
  int timeout_ms() const { return timeout_ms_; }
  int batch_chunk() const { return batch_chunk_; }

  // Make this device current on the calling thread; throws if poisoned.
  void enter();
  // Wait for `stream` to drain, polling at most timeout_ms; a timeout or a
  // CUDA error poisons the device. Then checks the kernels' error word.
  void sync(cudaStream_t stream);
  // Wait (bounded) for one recorded event.
  void wait_event(cudaEvent_t ev);
  // Throw (and poison) on a sticky CUDA error or a nonzero kernel error word
  // as last copied back by sync().
  void check_device_errors();
  void poison(const std::string& why) { poisoned_ = why.empty() ? "GPU failure" : why; }
  bool poisoned() const { return !poisoned_.empty(); }
  // Scratch of at least `bytes` for the launches queued on `stream` (the
  // GEMM's split-K partial sums): one buffer per stream, so that work on
  // concurrent streams never shares it; grows on demand.
  void* scratch(size_t bytes, cudaStream_t stream) {
    for (auto& e : scratch_)
      if (e.first == stream) {
        if (e.second.size() < bytes) {
          e.second.reserve(bytes);
          scratch_gen_++;
        }
        return e.second.get();
      }
    scratch_.emplace_back(stream, DeviceBuffer());
    scratch_.back().second.reserve(bytes);
    scratch_gen_++;
    return scratch_.back().second.get();
  }
  // Counts the scratch buffers' (re)allocations (a captured pass that used
  // an older one must not replay).
  uint64_t scratch_generation() const { return scratch_gen_; }

  // Launch timing (diagnostics, no counterpart in the reference): while it is
  // on, the kernels that report themselves record a CUDA event before and
  // after their launch on the stream they run on, with their name and
  // algorithmic FLOPs and bytes; models run their passes eagerly meanwhile.
  // Turning it on starts a new record.
  struct TimedLaunch {
    std::string name;
    double flop = 0, bytes = 0;
    cudaEvent_t a = nullptr, b = nullptr;
  };
  void set_timing(bool on);
  bool timing() const { return timing_; }
  // Record the start of a launch; returns its index, or -1 when off.
  int time_begin(const std::string& name, double flop, double bytes, cudaStream_t s);
  void time_end(int index, cudaStream_t s);
  const std::vector<TimedLaunch>& timed() const { return timed_; }
  // Waits for the recorded events; the duration of launch i in ms.
  float timed_ms(size_t i);

 private:
  int ordinal_ = 0;
  std::string name_;
  int sms_ = 0;
  int timeout_ms_ = 120000;
  int batch_chunk_ = 0;
  cudaStream_t stream_ = nullptr;
  cudaStream_t copy_stream_ = nullptr;
  DeviceBuffer dev_err_;
  std::vector<std::pair<cudaStream_t, DeviceBuffer>> scratch_;
  uint64_t scratch_gen_ = 0;
  PinnedBuffer host_err_;
  std::string poisoned_;
  bool timing_ = false;
  std::vector<TimedLaunch> timed_;
  std::vector<cudaEvent_t> event_pool_;
  size_t events_used_ = 0;
};


// RAII: make the device current for a call and restore the caller's.
// Model passes kept as CUDA graphs: hundreds of small launches replay with
// less per-launch cost. A pass runs eagerly the first time its key is seen
// (that run makes every allocation), is captured the second time and
// replayed after that. The key holds the shapes, the caller's buffers and
// the generations of the model's and the device's allocations, so a graph
// never replays over buffers that have moved; the four most recent keys
// keep their graphs. A pass that cannot be captured turns the graphs off
// for the model.
class PassGraph {
 public:
  ~PassGraph();
  void run(const std::vector<long long>& key, cudaStream_t s, const std::function<void(cudaStream_t)>& body);
  void reset();
  // a poisoned device: nothing is freed under possibly running work
  void leak() { entries_.clear(); }
  bool enabled = true;

 private:
  struct Entry {
    std::vector<long long> key;
    int seen = 0;
    cudaGraphExec_t exec = nullptr;
    uint64_t used = 0;
  };
  static constexpr size_t MAX_ENTRIES = 4;
  std::vector<Entry> entries_;
  uint64_t clock_ = 0;
};

class DeviceScope {
 public:
  explicit DeviceScope(Device& d);
  ~DeviceScope();

 private:
  int prev_ = -1;
  Device* prev_device_ = nullptr;
};

// While `on`, the side streams listed are the pass's own stream `main`
// (restored on scope exit): a pass whose launches are being timed runs them
// one after another, so each event pair measures one kernel alone.
class SerialStreams {
 public:
  SerialStreams(bool on, std::initializer_list<cudaStream_t*> side, cudaStream_t main) {
    if (!on) return;
    for (cudaStream_t* st : side) {
      saved_.emplace_back(st, *st);
      *st = main;
    }
  }
  ~SerialStreams() {
    for (auto& e : saved_) *e.first = e.second;
  }
  SerialStreams(const SerialStreams&) = delete;
  SerialStreams& operator=(const SerialStreams&) = delete;

 private:
  std::vector<std::pair<cudaStream_t*, cudaStream_t>> saved_;
};

// The device of the innermost DeviceScope on this thread (null outside one).
Device* scoped_device();

// Run `launch` (one kernel launch on `s`), recorded as `name` with its
// algorithmic FLOPs and bytes when the scoped device's launch timing is on.
template <class F>
void timed_launch(const char* name, double flop, double bytes, cudaStream_t s, F&& launch) {
  Device* d = scoped_device();
  const int t = d && d->timing() ? d->time_begin(name, flop, bytes, s) : -1;
  launch();
  if (t >= 0) d->time_end(t, s);
}

// Launch `kernel` as a programmatic dependent of the work before it on `s`:
// it may start while its predecessor drains, so it must execute
// griddepcontrol.wait (griddep_wait in sm100.cuh) before touching global
// memory.
template <class... KArgs, class... Args>
void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  IEC_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (so the
// library does not link libcuda and still loads on a machine without it).
void encode_tensor_map(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base,
                       const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box);

int device_count();

}  // namespace iec

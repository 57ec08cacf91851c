// Runtime layer: sessions, buffers, prepared programs of plan steps, events
// (ask_b200_runtime.h).  Semantics follow the reference Runtime
// (include/ask/Runtime/CUDA.h:66-175, lib/Runtime/CUDA.cpp:418-1005):
//   - one non-blocking stream per session; every call is serialised by the
//     session's recursive mutex (CUDA.cpp:192) and runs with the session's
//     device current, restoring the caller's device afterwards;
//   - prepareProgram checks the program structure, maps its internal buffers
//     to workspace slots and verifies the mapping (plan_check.h) before any
//     device work; submit validates every public port before enqueueing;
//   - a workspace (one set of slots, plus a CUDA graph in graph mode) is busy
//     from its submission until that submission's event completes; an idle
//     one is reused, otherwise a new one is allocated (CUDA.cpp:921-955) --
//     except that a program without internal buffers reuses its one
//     workspace while earlier submissions still run (stream order keeps its
//     graph's launches and updates apart), instead of building a new graph;
//   - counters: allocations, launches (steps enqueued), program_submissions,
//     workspace_reuses, prepared_internal_slots/bytes, graph_instantiations,
//     graph_launches, graph_nodes, graph_edges, graph_node_updates.
// A step is an ask_b200 plan (a recipe) or a loaded kernel (Session::load,
// CUDA.cpp:499-541: a cubin or PTX entry with declared parameter widths, such
// as the kernel artifacts of ask_b200_artifact.h); graph mode records each step
// (all of its kernels, and its pre-copy) as a child graph.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "ask_b200.h"
#include "ask_b200_runtime.h"
#include "json.h"
#include "plan_check.h"

extern "C" void askb_internal_set_error(const char* message);

namespace askb {
namespace rt {

namespace {

constexpr size_t kNone = SIZE_MAX;

struct Failure {
  int code;
  std::string message;
};

[[noreturn]] void fail(int code, const std::string& msg) { throw Failure{code, msg}; }
void require(bool ok, const std::string& msg) {
  if (!ok) fail(ASK_B200_E_INVALID, msg);
}
void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail(ASK_B200_E_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

template <class F>
int guarded(F&& body) {
  try {
    body();
    askb_internal_set_error("");
    return ASK_B200_OK;
  } catch (const Failure& f) {
    askb_internal_set_error(f.message.c_str());
    return f.code;
  } catch (const std::bad_alloc&) {
    askb_internal_set_error("host out of memory");
    return ASK_B200_E_INVALID;
  } catch (const std::exception& e) {
    askb_internal_set_error(e.what());
    return ASK_B200_E_INVALID;
  } catch (...) {
    askb_internal_set_error("unknown error");
    return ASK_B200_E_INVALID;
  }
}

void write_text(const std::string& s, char* buf, size_t cap, size_t* needed) {
  if (needed) *needed = s.size() + 1;
  if (buf && cap) {
    const size_t n = std::min(cap - 1, s.size());
    std::memcpy(buf, s.data(), n);
    buf[n] = '\0';
  }
}

// Makes the session's device current for the scope (the reference pushes the
// session's context around every driver call, lib/Runtime/CUDA.cpp:172-178).
class DeviceScope {
 public:
  explicit DeviceScope(int device) {
    cuda_check(cudaGetDevice(&prev_), "cudaGetDevice");
    if (prev_ != device) cuda_check(cudaSetDevice(device), "cudaSetDevice");
    changed_ = prev_ != device;
  }
  ~DeviceScope() {
    if (changed_) cudaSetDevice(prev_);
  }

 private:
  int prev_ = 0;
  bool changed_ = false;
};

struct EventImpl;
struct State;

// A loaded kernel (Session::load): a CUDA library holding the image and the
// entry's handle, with the parameter ABI it was checked against.
struct KernelImpl {
  const State* owner = nullptr;
  int device = 0;
  cudaLibrary_t lib = nullptr;
  cudaKernel_t fn = nullptr;
  std::string entry;
  std::vector<unsigned> widths;  // 0 = device pointer, else scalar bytes
  int max_threads = 0;
  int max_dynamic_shared = 0;
  ~KernelImpl() {
    if (lib) {
      int prev = 0;
      cudaGetDevice(&prev);
      cudaSetDevice(device);
      cudaLibraryUnload(lib);
      cudaSetDevice(prev);
    }
  }
};

struct State {
  int device = 0;
  cudaStream_t stream = nullptr;   // submissions
  cudaStream_t capture = nullptr;  // graph recording only
  std::recursive_mutex mu;
  bool closed = false;
  std::map<std::string, uint64_t> counters;
  std::vector<std::shared_ptr<EventImpl>> pending;
  std::map<std::pair<std::string, std::string>, std::shared_ptr<KernelImpl>> kernels;  // (image, entry)
  std::vector<cudaEvent_t> free_events;  // completion events of retired submissions, for reuse
  int major = 0, minor = 0;
  unsigned max_grid[3] = {0, 0, 0}, max_block[3] = {0, 0, 0}, max_threads = 0;
  ~State() {
    kernels.clear();
    if (stream || capture) {
      int prev = 0;
      cudaGetDevice(&prev);
      cudaSetDevice(device);
      for (cudaEvent_t e : free_events) cudaEventDestroy(e);
      if (stream) cudaStreamDestroy(stream);
      if (capture) cudaStreamDestroy(capture);
      cudaSetDevice(prev);
    }
  }
  void check_open() const { require(!closed, "session is closed"); }
};

struct Buffer {
  std::shared_ptr<State> st;
  uint64_t ptr = 0;
  size_t size = 0;
  bool readonly = false;
  bool owned = false;
  ~Buffer() {
    if (owned && ptr) {
      int prev = 0;
      cudaGetDevice(&prev);
      cudaSetDevice(st->device);
      cudaFree(reinterpret_cast<void*>(ptr));
      cudaSetDevice(prev);
    }
  }
};

std::shared_ptr<Buffer> allocate(const std::shared_ptr<State>& st, size_t bytes) {
  auto b = std::make_shared<Buffer>();
  b->st = st;
  b->size = bytes;
  b->owned = true;
  if (bytes) {
    void* p = nullptr;
    cuda_check(cudaMalloc(&p, bytes), "cudaMalloc");
    b->ptr = reinterpret_cast<uint64_t>(p);
  }
  ++st->counters["allocations"];
  return b;
}

struct Workspace {
  std::vector<std::shared_ptr<Buffer>> slots;
  bool busy = false;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  std::vector<cudaGraphNode_t> nodes;
  std::vector<std::vector<uint64_t>> recorded;  // per step: the addresses its child graph holds
  int device = 0;
  void drop_graph() {
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    exec = nullptr;
    graph = nullptr;
    nodes.clear();
    recorded.clear();
  }
  ~Workspace() {
    if (exec || graph) {
      int prev = 0;
      cudaGetDevice(&prev);
      cudaSetDevice(device);
      drop_graph();
      cudaSetDevice(prev);
    }
  }
};

struct PlanDeleter {
  void operator()(ask_b200_plan* p) const { ask_b200_plan_destroy(p); }
};

struct Step {
  std::shared_ptr<ask_b200_plan> plan;
  std::string kernel;
  std::vector<size_t> ports;  // logical buffers bound to the plan's inputs then outputs
  size_t n_inputs = 0;
  size_t scratch = kNone;     // private logical buffer for the plan's scratch
  size_t scratch_bytes = 0;
  bool copy = false;
  size_t copy_src = 0, copy_dst = 0;
  std::vector<size_t> touches;  // every buffer whose address the step's launch holds
  // A loaded-kernel step: one argument per parameter (a logical buffer, -1 for
  // null, or scalar ABI bytes) and a fixed launch.
  std::shared_ptr<KernelImpl> kern;
  std::vector<int64_t> arg_buffer;
  std::vector<std::string> arg_scalar;
  std::vector<uint64_t> arg_align;  // required address alignment of a pointer argument (1 = none)
  unsigned grid[3] = {1, 1, 1}, block[3] = {1, 1, 1}, shared = 0;
};

struct Program {
  std::weak_ptr<State> st;
  std::vector<size_t> sizes, inputs, outputs;
  std::vector<Step> steps;
  std::vector<size_t> slot_of;  // per logical buffer, kNone for public ports
  std::vector<size_t> capacity;
  std::vector<std::vector<size_t>> deps;
  std::vector<check::SlotAssignment> assignments;
  bool graph = false;
  size_t edges = 0;
  std::vector<size_t> allocated_outputs;                // output buffers that are not inputs
  std::vector<std::pair<size_t, size_t>> disjoint;      // (allocated output, other public port)
  std::vector<size_t> writable_ports;                   // output port positions that must be writable
  std::vector<std::shared_ptr<Workspace>> workspaces;
};

struct EventImpl {
  std::shared_ptr<State> st;
  cudaEvent_t ev = nullptr;
  bool finished = false;
  std::vector<std::shared_ptr<Buffer>> hold;
  std::shared_ptr<Workspace> ws;
  std::shared_ptr<Program> program;
  std::shared_ptr<KernelImpl> kernel;
  void finish() {
    if (ws) ws->busy = false;
    ws.reset();
    hold.clear();
    program.reset();
    kernel.reset();
    finished = true;
  }
  // The event goes back to the session's pool (the reference keeps retired
  // completion events for reuse, lib/Runtime/CUDA.cpp:554-564).
  ~EventImpl() {
    if (ev) {
      std::lock_guard<std::recursive_mutex> lock(st->mu);
      st->free_events.push_back(ev);
    }
  }
};

// A completion event from the session's pool, or a new one.
cudaEvent_t take_event(State& st) {
  if (!st.free_events.empty()) {
    cudaEvent_t e = st.free_events.back();
    st.free_events.pop_back();
    ++st.counters["event_reuses"];
    return e;
  }
  cudaEvent_t e = nullptr;
  cuda_check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
  ++st.counters["event_creations"];
  return e;
}

// Retire completed submissions (Session::reap).
void reap(State& s) {
  std::vector<std::shared_ptr<EventImpl>> keep;
  for (auto& e : s.pending) {
    if (e->finished) continue;
    const cudaError_t q = cudaEventQuery(e->ev);
    if (q == cudaSuccess) {
      e->finish();
    } else if (q == cudaErrorNotReady) {
      keep.push_back(e);
    } else {
      cuda_check(q, "cudaEventQuery");
    }
  }
  s.pending.swap(keep);
}

void synchronize(State& s) {
  cuda_check(cudaStreamSynchronize(s.stream), "cudaStreamSynchronize");
  for (auto& e : s.pending) e->finish();
  s.pending.clear();
}

// ---- loaded kernels (Session::load / validateLaunch / submit) -------------------
void check_types(const State& st, const std::vector<std::string>& types) {
  static const std::set<std::string> supported = {"bool", "i32", "i64", "f32", "f16", "bf16"};
  for (const std::string& t : types) {
    require(supported.count(t) != 0, "unsupported runtime element type: " + t);
    if (t == "bf16")
      require(st.major >= 8, "bf16 requires hardware support (CUDA compute capability >= 8.0); selected device has " +
                                 std::to_string(st.major) + "." + std::to_string(st.minor));
  }
}

// CUDA.cpp:499-541: validate the image, target and ABI, load the image once per
// (image, entry) and check the entry's parameter layout against the widths.
std::shared_ptr<KernelImpl> load_kernel(State& st, const std::string& image, const std::string& entry,
                                        const std::vector<std::string>& types, int arch,
                                        const std::vector<unsigned>& widths) {
  check_types(st, types);
  const bool ptx = image.compare(0, 4, "\x7f" "ELF") != 0;
  require(arch >= 10 && (ptx ? st.major * 10 + st.minor >= arch : st.major == arch / 10 && st.minor >= arch % 10),
          "CUDA code target is incompatible with the selected device");
  require(ptx ? image.find('\0') == std::string::npos && image.find(".version") != std::string::npos
              : image.size() >= 64,
          "runtime load requires a CUDA cubin ELF image or PTX text");
  require(!image.empty() && !entry.empty() && entry.find('\0') == std::string::npos,
          "kernel binary and entry must be nonempty");
  require(!widths.empty() && widths.size() <= 64, "unsupported kernel parameter count");
  for (unsigned w : widths) require(w == 0 || w == 1 || w == 2 || w == 4 || w == 8, "unsupported kernel parameter width");
  const auto key = std::make_pair(image, entry);
  const auto found = st.kernels.find(key);
  if (found != st.kernels.end()) {
    require(found->second->widths == widths, "cached kernel parameter contract differs");
    ++st.counters["module_hits"];
    return found->second;
  }
  auto k = std::make_shared<KernelImpl>();
  k->owner = &st;
  k->device = st.device;
  k->entry = entry;
  k->widths = widths;
  std::string data = image;
  if (ptx) data.push_back('\0');  // PTX is NUL-terminated driver input
  cuda_check(cudaLibraryLoadData(&k->lib, data.data(), nullptr, nullptr, 0, nullptr, nullptr, 0), "cudaLibraryLoadData");
  cuda_check(cudaLibraryGetKernel(&k->fn, k->lib, entry.c_str()), "cudaLibraryGetKernel");
  const void* f = reinterpret_cast<const void*>(k->fn);
  size_t expected = 0;
  for (size_t i = 0; i < widths.size(); ++i) {
    const size_t width = widths[i] ? widths[i] : sizeof(uint64_t);
    expected = (expected + width - 1) / width * width;
    size_t offset = 0, size = 0;
    const cudaError_t e = cudaFuncGetParamInfo(f, i, &offset, &size);
    if (e == cudaErrorInvalidValue) {  // fewer parameters than declared
      cudaGetLastError();
      fail(ASK_B200_E_INVALID, "kernel parameter count differs from the declared ABI");
    }
    cuda_check(e, "cudaFuncGetParamInfo");
    require(offset == expected && size == width, "kernel parameter layout differs from the declared ABI");
    expected += width;
  }
  size_t offset = 0, size = 0;
  const cudaError_t extra = cudaFuncGetParamInfo(f, widths.size(), &offset, &size);
  cudaGetLastError();  // the expected failure must not linger as the last error
  require(extra != cudaSuccess, "kernel parameter count differs from the declared ABI");
  cudaFuncAttributes attr{};
  cuda_check(cudaFuncGetAttributes(&attr, f), "cudaFuncGetAttributes");
  require(attr.maxThreadsPerBlock > 0 && attr.maxDynamicSharedSizeBytes >= 0, "invalid CUDA kernel resource limits");
  k->max_threads = attr.maxThreadsPerBlock;
  k->max_dynamic_shared = attr.maxDynamicSharedSizeBytes;
  st.kernels.emplace(key, k);
  ++st.counters["module_loads"];
  return k;
}

// CUDA.cpp:543-552.
void validate_launch(const State& st, const std::shared_ptr<KernelImpl>& k, const unsigned grid[3],
                     const unsigned block[3], unsigned shared) {
  require(k && k->owner == &st, "kernel belongs to a different CUDA execution session");
  require(shared <= unsigned(k->max_dynamic_shared), "dynamic shared memory exceeds the compiled kernel configured limit");
  uint64_t threads = 1;
  for (int i = 0; i < 3; ++i) {
    require(grid[i] && grid[i] <= st.max_grid[i], "launch grid exceeds device limits");
    require(block[i] && block[i] <= st.max_block[i], "launch block exceeds device limits");
    threads *= block[i];
  }
  require(threads <= st.max_threads && threads <= uint64_t(k->max_threads),
          "launch thread count exceeds kernel/device limits");
}

// Launch parameters: one 8-byte word per parameter holding the pointer or the
// scalar's little-endian ABI bytes.
void launch_kernel(const KernelImpl& k, std::vector<uint64_t>& words, const unsigned grid[3], const unsigned block[3],
                   unsigned shared, cudaStream_t stream) {
  std::vector<void*> params(words.size());
  for (size_t i = 0; i < words.size(); ++i) params[i] = &words[i];
  cuda_check(cudaLaunchKernel(reinterpret_cast<const void*>(k.fn), dim3(grid[0], grid[1], grid[2]),
                              dim3(block[0], block[1], block[2]), params.data(), shared, stream),
             "cudaLaunchKernel");
}

uint64_t scalar_word(const std::string& bytes) {
  uint64_t w = 0;
  std::memcpy(&w, bytes.data(), std::min(bytes.size(), sizeof w));
  return w;
}

std::string hex_bytes(const std::string& hex, const char* what) {
  require(hex.size() % 2 == 0, std::string(what) + " must be an even number of hex digits");
  std::string out;
  for (size_t i = 0; i < hex.size(); i += 2) {
    auto nib = [&](char c) -> int {
      if (c >= '0' && c <= '9') return c - '0';
      if (c >= 'a' && c <= 'f') return c - 'a' + 10;
      if (c >= 'A' && c <= 'F') return c - 'A' + 10;
      fail(ASK_B200_E_INVALID, std::string(what) + " must be hex digits");
    };
    out.push_back(char(nib(hex[i]) * 16 + nib(hex[i + 1])));
  }
  return out;
}

void dims3(const json::Value* v, unsigned out[3], const char* what) {
  require(v != nullptr, std::string("kernel step needs ") + what);
  const auto& a = v->as_array(what);
  require(a.size() == 3, std::string(what) + " must have three entries");
  for (int i = 0; i < 3; ++i) {
    const int64_t x = a[size_t(i)].as_int(what);
    require(x >= 1 && x <= 0xffffffffll, std::string(what) + " entries must be in [1, 2^32-1]");
    out[i] = unsigned(x);
  }
}

// A program step that launches a loaded kernel (PlanStep with `kernel`,
// CUDA.cpp:765-781): {"kernel": k, "inputs", "outputs", "grid", "block",
// "shared_bytes", "arguments": [{"buffer": b, "align": a} | {"buffer": -1} | {"scalar": "hex"}]}.
// "align" (optional, a power of two) is the address alignment the kernel
// needs for that pointer -- its element size; submissions binding a public
// buffer at another address are refused before anything is enqueued.
void prepare_kernel_step(const State& st, const json::Value& sv, const json::Value& kv,
                         const std::vector<std::shared_ptr<KernelImpl>>& kernels, const std::set<size_t>& ports,
                         Step& step) {
  const int64_t ki = kv.as_int("step kernel");
  require(ki >= 0 && size_t(ki) < kernels.size() && kernels[size_t(ki)], "program step kernel index is out of range");
  step.kern = kernels[size_t(ki)];
  step.kernel = step.kern->entry;
  dims3(sv.get("grid"), step.grid, "grid");
  dims3(sv.get("block"), step.block, "block");
  const json::Value* sh = sv.get("shared_bytes");
  const int64_t shared = sh ? sh->as_int("shared_bytes") : 0;
  require(shared >= 0 && shared <= 0xffffffffll, "shared_bytes must be in [0, 2^32-1]");
  step.shared = unsigned(shared);
  validate_launch(st, step.kern, step.grid, step.block, step.shared);
  const auto& args = sv.at("arguments").as_array("arguments");
  require(args.size() == step.kern->widths.size(), "program kernel argument count differs from its ABI");
  std::set<size_t> bound;
  for (size_t i = 0; i < args.size(); ++i) {
    const unsigned width = step.kern->widths[i];
    const json::Value* b = args[i].get("buffer");
    const json::Value* sc = args[i].get("scalar");
    const int64_t buffer = b ? b->as_int("argument buffer") : -1;
    const json::Value* al = args[i].get("align");
    const int64_t align = al ? al->as_int("argument align") : 1;
    require(align >= 1 && align <= 256 && (align & (align - 1)) == 0, "argument align must be a power of two up to 256");
    require(!al || !width, "scalar arguments take no alignment");
    const std::string bytes = sc ? hex_bytes(sc->as_str("argument scalar"), "argument scalar") : std::string();
    if (width) {
      require(buffer == -1 && sc && bytes.size() == width, "program scalar argument differs from its ABI");
    } else {
      require(!sc && buffer >= -1, "program pointer argument differs from its ABI");
      if (buffer >= 0) {
        require(ports.count(size_t(buffer)) != 0, "program argument is not a step port");
        bound.insert(size_t(buffer));
      }
    }
    step.arg_buffer.push_back(buffer);
    step.arg_scalar.push_back(bytes);
    step.arg_align.push_back(uint64_t(align));
  }
  require(bound == ports, "program step port is not bound to a kernel parameter");
}

// ---- program preparation --------------------------------------------------------
// Non-negative integers up to 2^64 - 1 (byte counts may use the full range).
std::vector<size_t> index_list(const json::Value& v, const char* what) {
  std::vector<size_t> out;
  for (const auto& x : v.as_array(what)) {
    const int64_t i = x.as_int(what);
    require(!x.negative, std::string(what) + " entries must be non-negative");
    out.push_back(size_t(uint64_t(i)));
  }
  return out;
}

// The reference partitions a row softmax into three owned steps (row max of
// cast(x), row sum of exp(cast(x) - max), normalise).  Three consecutive steps
// that are exactly those, bound as (x)->(m), (x, m)->(s), (x, m, s)->(y),
// become one fused softmax plan (softmax_kernels.cu) that still writes m, s
// and y: x is read once instead of three times and exp is computed once per
// element.  A program can opt out with "fuse": false.
void fuse_softmax(State& st, Program& p) {
  for (size_t i = 0; i + 2 < p.steps.size(); ++i) {
    const Step &a = p.steps[i], &b = p.steps[i + 1], &c = p.steps[i + 2];
    std::string dt;
    for (const char* t : {"f16", "bf16"})
      for (const char* red : {"reduce_warp_row_softmax_", "softmax_rows_"})
        for (const char* ew : {"ew_softmax_norm_", "softmax_rows_norm_"})
          if (a.kernel == std::string(red) + "max_" + t && b.kernel == std::string(red) + "sum_" + t &&
              c.kernel == std::string(ew) + t)
            dt = t;
    if (dt.empty() || a.copy || b.copy || c.copy || a.ports.size() != 2 || b.ports.size() != 3 || c.ports.size() != 4)
      continue;
    const size_t x = a.ports[0], m = a.ports[1], s = b.ports[2], y = c.ports[3];
    if (b.ports[0] != x || b.ports[1] != m || c.ports[0] != x || c.ports[1] != m || c.ports[2] != s) continue;
    const uint64_t rows = p.sizes[m] / 4, cols = rows ? p.sizes[x] / 2 / rows : 0;
    if (!rows || rows * cols * 2 != p.sizes[x]) continue;
    const std::string recipe = "{\"family\":\"softmax\",\"dtype\":\"" + dt + "\",\"rows\":" + std::to_string(rows) +
                               ",\"cols\":" + std::to_string(cols) + "}";
    ask_b200_plan* raw = nullptr;
    if (ask_b200_plan_create(recipe.c_str(), st.device, &raw) != ASK_B200_OK) continue;  // no fused kernel: keep 3 steps
    Step fused;
    fused.plan.reset(raw, PlanDeleter());
    fused.kernel = std::string("softmax_rows_") + dt;
    fused.ports = {x, m, s, y};
    fused.n_inputs = 1;
    p.steps.erase(p.steps.begin() + long(i), p.steps.begin() + long(i) + 3);
    p.steps.insert(p.steps.begin() + long(i), std::move(fused));
    ++st.counters["fused_softmax_steps"];
  }
}

std::shared_ptr<Program> prepare(const std::shared_ptr<State>& st, const char* text, bool graph,
                                 const std::vector<std::shared_ptr<KernelImpl>>& kernels) {
  require(text != nullptr, "program JSON is NULL");
  const json::Value root = json::Parser(text).parse();
  auto p = std::make_shared<Program>();
  p->st = st;
  p->sizes = index_list(root.at("buffer_sizes"), "buffer_sizes");
  p->inputs = index_list(root.at("inputs"), "inputs");
  p->outputs = index_list(root.at("outputs"), "outputs");
  require(!p->outputs.empty(), "program must have at least one output");
  const size_t declared = p->sizes.size();
  auto in_range = [&](size_t b) { require(b < declared, "program buffer index is out of range"); };
  std::set<size_t> available;
  for (size_t b : p->inputs) {
    in_range(b);
    require(available.insert(b).second, "program inputs must be unique");
  }
  for (size_t b : p->outputs) in_range(b);

  check::Allocation alloc;
  alloc.plan.public_inputs = p->inputs;
  alloc.plan.public_outputs = p->outputs;
  alloc.buffer_sizes = p->sizes;
  const json::Value* steps = root.get("steps");
  const std::vector<json::Value> none;
  for (const json::Value& sv : steps ? steps->as_array("steps") : none) {
    Step step;
    const std::vector<size_t> ins = index_list(sv.at("inputs"), "step inputs");
    const std::vector<size_t> outs = index_list(sv.at("outputs"), "step outputs");
    std::set<size_t> ports;
    for (size_t b : ins) {
      in_range(b);
      ports.insert(b);
    }
    for (size_t b : outs) {
      in_range(b);
      require(!available.count(b), "program step overwrites an existing logical buffer");
      require(ports.insert(b).second, "program step repeats or aliases an output");
    }
    step.ports = ins;
    step.ports.insert(step.ports.end(), outs.begin(), outs.end());
    step.n_inputs = ins.size();
    const json::Value* kv = sv.get("kernel");
    require(bool(kv) != bool(sv.get("recipe")), "program step requires one recipe or kernel");
    if (kv) {
      prepare_kernel_step(*st, sv, *kv, kernels, ports, step);
    } else {
      ask_b200_plan* raw = nullptr;
      const std::string& recipe = sv.at("recipe").as_str("step recipe");
      const int rc = ask_b200_plan_create(recipe.c_str(), st->device, &raw);
      if (rc != ASK_B200_OK) fail(rc, std::string("step recipe: ") + ask_b200_last_error());
      step.plan.reset(raw, PlanDeleter());
      size_t n_in = 0, n_out = 0, scratch = 0;
      ask_b200_plan_ports(raw, &n_in, &n_out);
      require(n_in == ins.size() && n_out == outs.size(),
              "step binds " + std::to_string(ins.size()) + " inputs and " + std::to_string(outs.size()) +
                  " outputs; its recipe has " + std::to_string(n_in) + " and " + std::to_string(n_out));
      size_t needed = 0;
      ask_b200_plan_describe(raw, nullptr, 0, &needed);
      std::string desc(needed, '\0');
      ask_b200_plan_describe(raw, &desc[0], needed, &needed);
      const json::Value d = json::Parser(desc.c_str()).parse();
      step.kernel = d.at("kernel").as_str("kernel");
      const auto& pm = d.at("port_map").as_array("port_map");
      for (size_t k = 0; k < pm.size(); ++k) {
        const uint64_t bytes = uint64_t(pm[k].at("elements").as_int("elements")) *
                               uint64_t(pm[k].at("storage_bytes").as_int("storage_bytes"));
        require(p->sizes[step.ports[k]] == bytes,
                "step port " + std::to_string(k) + " needs " + std::to_string(bytes) + " bytes; logical buffer " +
                    std::to_string(step.ports[k]) + " has " + std::to_string(p->sizes[step.ports[k]]));
      }
      ask_b200_plan_scratch_bytes(raw, &scratch);
      step.scratch_bytes = scratch;
    }
    if (const json::Value* pc = sv.get("pre_copy")) {
      const int64_t src = pc->at("source").as_int("pre_copy source"), dst = pc->at("destination").as_int("pre_copy destination");
      require(src >= 0 && dst >= 0 && size_t(src) < declared && size_t(dst) < declared,
              "pre-copy buffer index is out of range");
      require(p->sizes[size_t(src)] == p->sizes[size_t(dst)], "pre-copy buffer sizes must match");
      require(ports.count(size_t(src)) && ports.count(size_t(dst)), "pre-copy buffers must be ports of the step");
      step.copy = true;
      step.copy_src = size_t(src);
      step.copy_dst = size_t(dst);
    }
    available.insert(outs.begin(), outs.end());
    p->steps.push_back(std::move(step));
  }
  require(available.size() == declared, "program contains an undefined buffer");
  const json::Value* fuse = root.get("fuse");
  if (!fuse || fuse->kind != json::Value::Bool || fuse->b) fuse_softmax(*st, *p);
  for (Step& step : p->steps) {
    check::StepPorts sp;
    sp.inputs.assign(step.ports.begin(), step.ports.begin() + long(step.n_inputs));
    sp.outputs.assign(step.ports.begin() + long(step.n_inputs), step.ports.end());
    if (step.scratch_bytes) {  // a private logical buffer with this step's lifetime
      step.scratch = alloc.buffer_sizes.size();
      sp.outputs.push_back(step.scratch);
      alloc.buffer_sizes.push_back(step.scratch_bytes);
    }
    step.touches = step.ports;
    if (step.scratch != kNone) step.touches.push_back(step.scratch);
    alloc.plan.steps.push_back(sp);
  }
  alloc.plan.buffer_count = alloc.buffer_sizes.size();
  if (graph)
    check::assign_graph_slots(alloc);
  else
    check::assign_stream_slots(alloc);
  const check::Verdict v = check::check_allocation(alloc);
  require(v.pass, "ASK execution plan validation failed: " + v.explanation);

  p->graph = graph && !p->steps.empty();
  p->deps = alloc.dependencies;
  for (const auto& d : p->deps) p->edges += d.size();
  p->capacity = alloc.slot_capacity_bytes;
  p->assignments = alloc.assignments;
  p->slot_of.assign(alloc.plan.buffer_count, kNone);
  for (const auto& a : alloc.assignments) p->slot_of[a.buffer] = a.slot;
  p->sizes = alloc.buffer_sizes;  // including the scratch buffers
  std::set<size_t> pub(p->inputs.begin(), p->inputs.end());
  pub.insert(p->outputs.begin(), p->outputs.end());
  for (size_t o : std::set<size_t>(p->outputs.begin(), p->outputs.end())) {
    if (std::find(p->inputs.begin(), p->inputs.end(), o) != p->inputs.end()) continue;
    p->allocated_outputs.push_back(o);
    for (size_t other : pub)
      if (other != o) p->disjoint.emplace_back(o, other);
  }
  for (size_t k = 0; k < p->outputs.size(); ++k)
    if (std::find(p->allocated_outputs.begin(), p->allocated_outputs.end(), p->outputs[k]) != p->allocated_outputs.end())
      p->writable_ports.push_back(k);
  st->counters["prepared_internal_slots"] += p->capacity.size();
  for (size_t c : p->capacity) st->counters["prepared_internal_bytes"] += c;
  return p;
}

std::string describe(const Program& p) {
  std::ostringstream o;
  auto list = [&](const std::vector<size_t>& v) {
    o << "[";
    for (size_t i = 0; i < v.size(); ++i) o << (i ? "," : "") << v[i];
    o << "]";
  };
  o << "{\"graph\":" << (p.graph ? "true" : "false") << ",\"buffer_sizes\":";
  list(p.sizes);
  o << ",\"slot_capacity_bytes\":";
  list(p.capacity);
  o << ",\"assignments\":[";
  for (size_t i = 0; i < p.assignments.size(); ++i)
    o << (i ? "," : "") << "[" << p.assignments[i].buffer << "," << p.assignments[i].slot << "]";
  o << "],\"dependencies\":[";
  for (size_t i = 0; i < p.deps.size(); ++i) {
    o << (i ? "," : "");
    list(p.deps[i]);
  }
  o << "],\"steps\":[";
  for (size_t i = 0; i < p.steps.size(); ++i) {
    const Step& s = p.steps[i];
    o << (i ? "," : "") << "{\"kernel\":\"" << s.kernel << "\",\"ports\":";
    list(s.ports);
    o << ",\"scratch\":";
    if (s.scratch == kNone) o << "null"; else o << s.scratch;
    o << "}";
  }
  o << "]}";
  return o.str();
}

// ---- submission -----------------------------------------------------------------
// Addresses of every logical buffer for one submission on one workspace.
std::vector<uint64_t> addresses(const Program& p, const std::vector<std::shared_ptr<Buffer>>& bound,
                                const Workspace& ws) {
  std::vector<uint64_t> a(p.sizes.size(), 0);
  for (size_t b = 0; b < a.size(); ++b)
    a[b] = p.slot_of[b] == kNone ? (bound[b] ? bound[b]->ptr : 0) : ws.slots[p.slot_of[b]]->ptr;
  return a;
}

void enqueue_step(const Program& p, const Step& s, const std::vector<uint64_t>& addr, cudaStream_t stream) {
  if (s.copy && addr[s.copy_src] != addr[s.copy_dst] && p.sizes[s.copy_dst])
    cuda_check(cudaMemcpyAsync(reinterpret_cast<void*>(addr[s.copy_dst]), reinterpret_cast<const void*>(addr[s.copy_src]),
                               p.sizes[s.copy_dst], cudaMemcpyDeviceToDevice, stream),
               "pre-copy");
  if (s.kern) {
    std::vector<uint64_t> words(s.arg_buffer.size());
    for (size_t i = 0; i < words.size(); ++i)
      words[i] = s.kern->widths[i] ? scalar_word(s.arg_scalar[i]) : s.arg_buffer[i] >= 0 ? addr[size_t(s.arg_buffer[i])] : 0;
    launch_kernel(*s.kern, words, s.grid, s.block, s.shared, stream);
    return;
  }
  std::vector<uint64_t> ports(s.ports.size());
  for (size_t k = 0; k < ports.size(); ++k) ports[k] = addr[s.ports[k]];
  const uint64_t scratch = s.scratch == kNone ? 0 : addr[s.scratch];
  const int rc = ask_b200_plan_launch(s.plan.get(), ports.data(), ports.size(), scratch, stream);
  if (rc != ASK_B200_OK) fail(rc, std::string("step ") + s.kernel + ": " + ask_b200_last_error());
}

std::vector<uint64_t> step_addresses(const Step& s, const std::vector<uint64_t>& addr) {
  std::vector<uint64_t> v;
  for (size_t b : s.touches) v.push_back(addr[b]);
  if (s.copy) {
    v.push_back(addr[s.copy_src]);
    v.push_back(addr[s.copy_dst]);
  }
  return v;
}

cudaGraph_t record_step(State& st, const Program& p, const Step& s, const std::vector<uint64_t>& addr) {
  cuda_check(cudaStreamBeginCapture(st.capture, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
  try {
    enqueue_step(p, s, addr, st.capture);
  } catch (...) {
    cudaGraph_t g = nullptr;
    cudaStreamEndCapture(st.capture, &g);
    if (g) cudaGraphDestroy(g);
    throw;
  }
  cudaGraph_t g = nullptr;
  cuda_check(cudaStreamEndCapture(st.capture, &g), "cudaStreamEndCapture");
  return g;
}

void build_graph(State& st, const Program& p, Workspace& ws, const std::vector<uint64_t>& addr) {
  ws.drop_graph();
  cuda_check(cudaGraphCreate(&ws.graph, 0), "cudaGraphCreate");
  std::vector<cudaGraphNode_t> deps;
  for (size_t i = 0; i < p.steps.size(); ++i) {
    cudaGraph_t child = record_step(st, p, p.steps[i], addr);
    deps.clear();
    for (size_t d : p.deps[i]) deps.push_back(ws.nodes[d]);
    cudaGraphNode_t node = nullptr;
    const cudaError_t e = cudaGraphAddChildGraphNode(&node, ws.graph, deps.data(), deps.size(), child);
    cudaGraphDestroy(child);  // the node holds its own copy
    cuda_check(e, "cudaGraphAddChildGraphNode");
    ws.nodes.push_back(node);
    ws.recorded.push_back(step_addresses(p.steps[i], addr));
  }
  cuda_check(cudaGraphInstantiate(&ws.exec, ws.graph, 0), "cudaGraphInstantiate");
  ++st.counters["graph_instantiations"];
  st.counters["graph_nodes"] += p.steps.size();
  st.counters["graph_edges"] += p.edges;
}

// Re-record the steps whose addresses changed; a step whose new recording has
// another shape (a plan may pick other kernels for aliased ports) rebuilds
// the whole executable graph.
void update_graph(State& st, const Program& p, Workspace& ws, const std::vector<uint64_t>& addr) {
  for (size_t i = 0; i < p.steps.size(); ++i) {
    std::vector<uint64_t> now = step_addresses(p.steps[i], addr);
    if (now == ws.recorded[i]) continue;
    cudaGraph_t child = record_step(st, p, p.steps[i], addr);
    const cudaError_t e = cudaGraphExecChildGraphNodeSetParams(ws.exec, ws.nodes[i], child);
    cudaGraphDestroy(child);
    if (e != cudaSuccess) {
      cudaGetLastError();  // clear the update error and start over
      build_graph(st, p, ws, addr);
      return;
    }
    ws.recorded[i] = std::move(now);
    ++st.counters["graph_node_updates"];
  }
}

std::shared_ptr<EventImpl> enqueue(const std::shared_ptr<State>& stp, const std::shared_ptr<Program>& pp,
                                   std::vector<std::shared_ptr<Buffer>> bound) {
  State& st = *stp;
  Program& p = *pp;
  std::shared_ptr<Workspace> ws;
  auto idle = [&] {
    for (const auto& w : p.workspaces)
      if (!w->busy) return w;
    return std::shared_ptr<Workspace>();
  };
  ws = idle();
  // A program without internal buffers keeps one workspace: nothing of an
  // earlier submission lives in it but its graph, and a graph is launched and
  // updated in stream order (an update affects later launches only), so a
  // submission need not wait for -- or rebuild beside -- one still running.
  if (!ws && p.capacity.empty() && !p.workspaces.empty()) ws = p.workspaces.front();
  if (!ws || st.pending.size() >= 64) {
    reap(st);
    if (!ws) ws = idle();
  }
  if (ws) {
    ++st.counters["workspace_reuses"];
  } else {
    auto fresh = std::make_shared<Workspace>();
    fresh->device = st.device;
    for (size_t c : p.capacity) fresh->slots.push_back(allocate(stp, c));
    p.workspaces.push_back(fresh);
    ws = fresh;
  }
  const std::vector<uint64_t> addr = addresses(p, bound, *ws);
  auto ev = std::make_shared<EventImpl>();
  ev->st = stp;
  ev->ev = take_event(st);
  try {
    if (p.graph) {
      if (!ws->exec)
        build_graph(st, p, *ws, addr);
      else
        update_graph(st, p, *ws, addr);
      cuda_check(cudaGraphLaunch(ws->exec, st.stream), "cudaGraphLaunch");
      ++st.counters["graph_launches"];
      st.counters["launches"] += p.steps.size();
    } else {
      for (const Step& s : p.steps) {
        enqueue_step(p, s, addr, st.stream);
        ++st.counters["launches"];
      }
    }
    cuda_check(cudaEventRecord(ev->ev, st.stream), "cudaEventRecord");
  } catch (...) {
    // Steps before the failing one may be queued: keep every buffer alive
    // until the stream has drained them.
    cudaStreamSynchronize(st.stream);
    throw;
  }
  ev->hold = std::move(bound);
  ev->ws = ws;
  ev->program = pp;
  ws->busy = true;
  st.pending.push_back(ev);
  ++st.counters["program_submissions"];
  return ev;
}

void bind(const Program& p, std::vector<std::shared_ptr<Buffer>>& bound, size_t index,
          const std::shared_ptr<Buffer>& b, const std::shared_ptr<State>& st) {
  require(b && b->st == st, "program tensor belongs to a different CUDA execution session");
  require(b->size == p.sizes[index], "program tensor byte count differs from its compiled type");
  require(!bound[index] || bound[index]->ptr == b->ptr, "repeated logical buffers must use the same device storage");
  bound[index] = b;
}

std::shared_ptr<EventImpl> submit(const std::shared_ptr<Program>& pp, const std::vector<std::shared_ptr<Buffer>>& ins,
                                  const std::vector<std::shared_ptr<Buffer>>& outs) {
  std::shared_ptr<State> st = pp->st.lock();
  require(bool(st), "program execution session no longer exists");
  std::lock_guard<std::recursive_mutex> lock(st->mu);
  st->check_open();
  DeviceScope scope(st->device);
  const Program& p = *pp;
  require(ins.size() == p.inputs.size() && outs.size() == p.outputs.size(),
          "program input/output count differs from its contract");
  std::vector<std::shared_ptr<Buffer>> bound(p.sizes.size());
  for (size_t i = 0; i < ins.size(); ++i) bind(p, bound, p.inputs[i], ins[i], st);
  for (size_t i = 0; i < outs.size(); ++i) bind(p, bound, p.outputs[i], outs[i], st);
  for (size_t k : p.writable_ports) require(!outs[k]->readonly, "program output tensor is read-only");
  for (const auto& [o, other] : p.disjoint) {
    const Buffer& a = *bound[o];
    const Buffer& b = *bound[other];
    require(!a.size || !b.size || a.ptr + a.size <= b.ptr || b.ptr + b.size <= a.ptr,
            "distinct program output buffers must not overlap other ports");
  }
  for (const Step& s : p.steps)
    for (size_t i = 0; i < s.arg_align.size(); ++i) {
      const int64_t b = s.arg_buffer[i];
      if (b >= 0 && bound[size_t(b)] && bound[size_t(b)]->ptr % s.arg_align[i])
        fail(ASK_B200_E_INVALID, "kernel step " + s.kernel + " argument " + std::to_string(i) +
                                     " is not aligned to " + std::to_string(s.arg_align[i]) + " bytes");
    }
  return enqueue(st, pp, std::move(bound));
}

std::shared_ptr<EventImpl> run(const std::shared_ptr<Program>& pp, const std::vector<std::shared_ptr<Buffer>>& ins,
                               std::vector<std::shared_ptr<Buffer>>& outs) {
  std::shared_ptr<State> st = pp->st.lock();
  require(bool(st), "program execution session no longer exists");
  std::lock_guard<std::recursive_mutex> lock(st->mu);
  st->check_open();
  DeviceScope scope(st->device);
  const Program& p = *pp;
  require(ins.size() == p.inputs.size(), "program input/output count differs from its contract");
  std::vector<std::shared_ptr<Buffer>> bound(p.sizes.size());
  for (size_t i = 0; i < ins.size(); ++i) bind(p, bound, p.inputs[i], ins[i], st);  // before any allocation
  outs.assign(p.outputs.size(), nullptr);
  for (size_t k = 0; k < p.outputs.size(); ++k) {
    const size_t o = p.outputs[k];
    if (!bound[o]) bound[o] = allocate(st, p.sizes[o]);
    outs[k] = bound[o];
  }
  return submit(pp, ins, outs);
}

}  // namespace
}  // namespace rt
}  // namespace askb

// ---- C ABI ----------------------------------------------------------------------
using namespace askb;
using namespace askb::rt;

struct ask_b200_session {
  std::shared_ptr<State> st;
};
struct ask_b200_buffer {
  std::shared_ptr<Buffer> b;
};
struct ask_b200_program {
  std::shared_ptr<Program> p;
};
struct ask_b200_event {
  std::shared_ptr<EventImpl> e;
};
struct ask_b200_kernel {
  std::shared_ptr<KernelImpl> k;
};

namespace {

State& session_state(ask_b200_session* s) {
  require(s && s->st, "session is NULL");
  return *s->st;
}

std::vector<std::shared_ptr<Buffer>> buffers(ask_b200_buffer* const* list, size_t n) {
  require(n == 0 || list, "buffer list is NULL");
  std::vector<std::shared_ptr<Buffer>> out(n);
  for (size_t i = 0; i < n; ++i) out[i] = list[i] ? list[i]->b : nullptr;
  return out;
}

check::Plan parse_check_plan(const json::Value& v) {
  check::Plan p;
  p.buffer_count = size_t(v.at("buffer_count").as_int("buffer_count"));
  p.public_inputs = index_list(v.at("public_inputs"), "public_inputs");
  p.public_outputs = index_list(v.at("public_outputs"), "public_outputs");
  for (const auto& s : v.at("steps").as_array("steps"))
    p.steps.push_back({index_list(s.at("inputs"), "step inputs"), index_list(s.at("outputs"), "step outputs")});
  return p;
}

}  // namespace

extern "C" {

int ask_b200_session_create(int device, ask_b200_session** out) {
  return guarded([&] {
    require(out != nullptr, "out is NULL");
    *out = nullptr;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count)
      fail(ASK_B200_E_DEVICE, "no CUDA device " + std::to_string(device));
    auto st = std::make_shared<State>();
    st->device = device;
    DeviceScope scope(device);
    cudaDeviceProp prop{};
    cuda_check(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    st->major = prop.major;
    st->minor = prop.minor;
    for (int i = 0; i < 3; ++i) {
      st->max_grid[i] = unsigned(prop.maxGridSize[i]);
      st->max_block[i] = unsigned(prop.maxThreadsDim[i]);
    }
    st->max_threads = unsigned(prop.maxThreadsPerBlock);
    cuda_check(cudaStreamCreateWithFlags(&st->stream, cudaStreamNonBlocking), "cudaStreamCreate");
    cuda_check(cudaStreamCreateWithFlags(&st->capture, cudaStreamNonBlocking), "cudaStreamCreate");
    for (const char* k : {"allocations", "launches", "program_submissions", "workspace_reuses", "prepared_internal_slots",
                          "prepared_internal_bytes", "graph_instantiations", "graph_launches", "graph_nodes",
                          "graph_edges", "graph_node_updates", "fused_softmax_steps", "module_loads", "module_hits", "event_creations",
                          "event_reuses"})
      st->counters[k] = 0;
    *out = new ask_b200_session{st};
  });
}

int ask_b200_session_release(ask_b200_session* s) {
  if (!s) return ASK_B200_OK;
  const int rc = guarded([&] {
    State& st = session_state(s);
    std::lock_guard<std::recursive_mutex> lock(st.mu);
    if (!st.closed) {
      DeviceScope scope(st.device);
      synchronize(st);
      st.closed = true;
    }
  });
  delete s;
  return rc;
}

int ask_b200_session_synchronize(ask_b200_session* s) {
  return guarded([&] {
    State& st = session_state(s);
    std::lock_guard<std::recursive_mutex> lock(st.mu);
    st.check_open();
    DeviceScope scope(st.device);
    synchronize(st);
  });
}

int ask_b200_session_reap(ask_b200_session* s) {
  return guarded([&] {
    State& st = session_state(s);
    std::lock_guard<std::recursive_mutex> lock(st.mu);
    DeviceScope scope(st.device);
    reap(st);
  });
}

int ask_b200_session_stream(ask_b200_session* s, void** stream) {
  return guarded([&] {
    require(stream != nullptr, "stream is NULL");
    *stream = session_state(s).stream;
  });
}

int ask_b200_session_wait_stream(ask_b200_session* s, void* stream) {
  return guarded([&] {
    State& st = session_state(s);
    std::lock_guard<std::recursive_mutex> lock(st.mu);
    st.check_open();
    DeviceScope scope(st.device);
    cudaEvent_t e = nullptr;
    cuda_check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
    cudaError_t r = cudaEventRecord(e, static_cast<cudaStream_t>(stream));
    if (r == cudaSuccess) r = cudaStreamWaitEvent(st.stream, e, 0);
    cudaEventDestroy(e);
    cuda_check(r, "waiting for the external stream");
  });
}

int ask_b200_session_stats(ask_b200_session* s, char* buf, size_t cap, size_t* needed) {
  return guarded([&] {
    State& st = session_state(s);
    std::lock_guard<std::recursive_mutex> lock(st.mu);
    std::ostringstream o;
    o << "{";
    bool first = true;
    for (const auto& [k, v] : st.counters) {
      o << (first ? "" : ",") << "\"" << k << "\":" << v;
      first = false;
    }
    o << "}";
    write_text(o.str(), buf, cap, needed);
  });
}

int ask_b200_buffer_allocate(ask_b200_session* s, size_t bytes, ask_b200_buffer** out) {
  return guarded([&] {
    require(out != nullptr, "out is NULL");
    *out = nullptr;
    State& st = session_state(s);
    std::lock_guard<std::recursive_mutex> lock(st.mu);
    st.check_open();
    DeviceScope scope(st.device);
    *out = new ask_b200_buffer{allocate(s->st, bytes)};
  });
}

int ask_b200_buffer_import(ask_b200_session* s, uint64_t pointer, size_t bytes, int readonly, ask_b200_buffer** out) {
  return guarded([&] {
    require(out != nullptr, "out is NULL");
    *out = nullptr;
    State& st = session_state(s);
    std::lock_guard<std::recursive_mutex> lock(st.mu);
    st.check_open();
    require(pointer != 0 || bytes == 0, "imported buffer address is NULL");
    auto b = std::make_shared<Buffer>();
    b->st = s->st;
    b->ptr = pointer;
    b->size = bytes;
    b->readonly = readonly != 0;
    *out = new ask_b200_buffer{b};
  });
}

int ask_b200_buffer_info(const ask_b200_buffer* b, uint64_t* pointer, size_t* bytes, int* readonly) {
  return guarded([&] {
    require(b && b->b, "buffer is NULL");
    if (pointer) *pointer = b->b->ptr;
    if (bytes) *bytes = b->b->size;
    if (readonly) *readonly = b->b->readonly ? 1 : 0;
  });
}

int ask_b200_buffer_copy_from_host(ask_b200_buffer* b, const void* src, size_t bytes) {
  return guarded([&] {
    require(b && b->b, "buffer is NULL");
    Buffer& buf = *b->b;
    require(!buf.readonly, "buffer is read-only");
    require(bytes == buf.size, "host copy size differs from the buffer size");
    require(bytes == 0 || src, "source is NULL");
    std::lock_guard<std::recursive_mutex> lock(buf.st->mu);
    DeviceScope scope(buf.st->device);
    if (bytes) {
      cuda_check(cudaMemcpyAsync(reinterpret_cast<void*>(buf.ptr), src, bytes, cudaMemcpyHostToDevice, buf.st->stream),
                 "copy to device");
      cuda_check(cudaStreamSynchronize(buf.st->stream), "cudaStreamSynchronize");
    }
  });
}

int ask_b200_buffer_copy_to_host(const ask_b200_buffer* b, void* dst, size_t bytes) {
  return guarded([&] {
    require(b && b->b, "buffer is NULL");
    const Buffer& buf = *b->b;
    require(bytes == buf.size, "host copy size differs from the buffer size");
    require(bytes == 0 || dst, "destination is NULL");
    std::lock_guard<std::recursive_mutex> lock(buf.st->mu);
    DeviceScope scope(buf.st->device);
    if (bytes) {
      cuda_check(cudaMemcpyAsync(dst, reinterpret_cast<const void*>(buf.ptr), bytes, cudaMemcpyDeviceToHost, buf.st->stream),
                 "copy to host");
      cuda_check(cudaStreamSynchronize(buf.st->stream), "cudaStreamSynchronize");
    }
  });
}

int ask_b200_buffer_release(ask_b200_buffer* b) {
  delete b;
  return ASK_B200_OK;
}

int ask_b200_program_prepare(ask_b200_session* s, const char* program_json, int graph, ask_b200_program** out) {
  return guarded([&] {
    require(out != nullptr, "out is NULL");
    *out = nullptr;
    State& st = session_state(s);
    std::lock_guard<std::recursive_mutex> lock(st.mu);
    st.check_open();
    DeviceScope scope(st.device);
    *out = new ask_b200_program{prepare(s->st, program_json, graph != 0, {})};
  });
}

int ask_b200_program_prepare_kernels(ask_b200_session* s, const char* program_json, ask_b200_kernel* const* kernels,
                                     size_t n_kernels, int graph, ask_b200_program** out) {
  return guarded([&] {
    require(out != nullptr, "out is NULL");
    *out = nullptr;
    require(n_kernels == 0 || kernels, "kernel list is NULL");
    State& st = session_state(s);
    std::lock_guard<std::recursive_mutex> lock(st.mu);
    st.check_open();
    DeviceScope scope(st.device);
    std::vector<std::shared_ptr<KernelImpl>> ks(n_kernels);
    for (size_t i = 0; i < n_kernels; ++i) ks[i] = kernels[i] ? kernels[i]->k : nullptr;
    *out = new ask_b200_program{prepare(s->st, program_json, graph != 0, ks)};
  });
}

int ask_b200_kernel_load(ask_b200_session* s, const void* image, size_t bytes, const char* entry,
                         const char* const* required_types, size_t n_types, int arch, const unsigned* widths,
                         size_t n_widths, ask_b200_kernel** out) {
  return guarded([&] {
    require(out != nullptr, "out is NULL");
    *out = nullptr;
    require(image || !bytes, "kernel image is NULL");
    require(entry != nullptr, "kernel entry is NULL");
    require(n_types == 0 || required_types, "required type list is NULL");
    require(n_widths == 0 || widths, "parameter width list is NULL");
    State& st = session_state(s);
    std::lock_guard<std::recursive_mutex> lock(st.mu);
    st.check_open();
    DeviceScope scope(st.device);
    std::vector<std::string> types;
    for (size_t i = 0; i < n_types; ++i) {
      require(required_types[i] != nullptr, "required type is NULL");
      types.emplace_back(required_types[i]);
    }
    const std::string img(static_cast<const char*>(image), bytes);
    *out = new ask_b200_kernel{load_kernel(st, img, entry, types, arch, std::vector<unsigned>(widths, widths + n_widths))};
  });
}

int ask_b200_kernel_info(const ask_b200_kernel* k, char* entry, size_t cap, size_t* needed, unsigned* max_threads) {
  return guarded([&] {
    require(k && k->k, "kernel is NULL");
    if (max_threads) *max_threads = unsigned(k->k->max_threads);
    write_text(k->k->entry, entry, cap, needed);
  });
}

int ask_b200_kernel_release(ask_b200_kernel* k) {
  delete k;
  return ASK_B200_OK;
}

int ask_b200_kernel_submit(ask_b200_session* s, ask_b200_kernel* k, const ask_b200_kernel_arg* args, size_t n_args,
                           const unsigned grid[3], const unsigned block[3], unsigned shared_bytes, ask_b200_event** event) {
  return guarded([&] {
    require(event != nullptr, "event is NULL");
    *event = nullptr;
    require(k && k->k, "kernel is NULL");
    require(grid && block, "grid or block is NULL");
    require(n_args == 0 || args, "argument list is NULL");
    State& st = session_state(s);
    std::lock_guard<std::recursive_mutex> lock(st.mu);
    st.check_open();
    DeviceScope scope(st.device);
    const KernelImpl& kern = *k->k;
    validate_launch(st, k->k, grid, block, shared_bytes);
    require(n_args == kern.widths.size(), "kernel argument count differs from its ABI");
    std::vector<uint64_t> words(n_args, 0);
    std::vector<std::shared_ptr<Buffer>> hold;
    for (size_t i = 0; i < n_args; ++i) {
      const unsigned width = kern.widths[i];
      if (width) {
        require(!args[i].buffer && args[i].scalar && args[i].scalar_bytes == width,
                "scalar argument byte width differs from its ABI");
        std::memcpy(&words[i], args[i].scalar, width);
      } else {
        require(!args[i].scalar && !args[i].scalar_bytes, "pointer argument requires a device buffer or null");
        if (args[i].buffer) {
          require(args[i].buffer->b && args[i].buffer->b->st == s->st,
                  "device tensor belongs to a different CUDA execution session");
          require(args[i].align <= 1 || args[i].buffer->b->ptr % args[i].align == 0,
                  "kernel argument " + std::to_string(i) + " is not aligned to " + std::to_string(args[i].align) +
                      " bytes");
          words[i] = args[i].buffer->b->ptr;
          hold.push_back(args[i].buffer->b);
        }
      }
    }
    reap(st);
    auto ev = std::make_shared<EventImpl>();
    ev->st = s->st;
    ev->ev = take_event(st);
    launch_kernel(kern, words, grid, block, shared_bytes, st.stream);
    ++st.counters["launches"];
    cuda_check(cudaEventRecord(ev->ev, st.stream), "cudaEventRecord");
    ev->hold = std::move(hold);
    ev->kernel = k->k;
    st.pending.push_back(ev);
    *event = new ask_b200_event{ev};
  });
}

int ask_b200_program_describe(const ask_b200_program* p, char* buf, size_t cap, size_t* needed) {
  return guarded([&] {
    require(p && p->p, "program is NULL");
    write_text(describe(*p->p), buf, cap, needed);
  });
}

int ask_b200_program_submit(ask_b200_program* p, ask_b200_buffer* const* inputs, size_t n_inputs,
                            ask_b200_buffer* const* outputs, size_t n_outputs, ask_b200_event** event) {
  return guarded([&] {
    require(p && p->p, "program is NULL");
    require(event != nullptr, "event is NULL");
    *event = nullptr;
    auto e = submit(p->p, buffers(inputs, n_inputs), buffers(outputs, n_outputs));
    *event = new ask_b200_event{e};
  });
}

int ask_b200_program_run(ask_b200_program* p, ask_b200_buffer* const* inputs, size_t n_inputs, ask_b200_buffer** outputs,
                         size_t n_outputs, ask_b200_event** event) {
  return guarded([&] {
    require(p && p->p, "program is NULL");
    require(event != nullptr && (outputs != nullptr || n_outputs == 0), "outputs or event is NULL");
    *event = nullptr;
    require(n_outputs == p->p->outputs.size(), "program input/output count differs from its contract");
    std::vector<std::shared_ptr<Buffer>> outs;
    auto e = run(p->p, buffers(inputs, n_inputs), outs);
    for (size_t k = 0; k < n_outputs; ++k) outputs[k] = new ask_b200_buffer{outs[k]};
    *event = new ask_b200_event{e};
  });
}

int ask_b200_program_release(ask_b200_program* p) {
  delete p;
  return ASK_B200_OK;
}

int ask_b200_event_query(ask_b200_event* e, int* done) {
  return guarded([&] {
    require(e && e->e, "event is NULL");
    require(done != nullptr, "done is NULL");
    EventImpl& ev = *e->e;
    std::lock_guard<std::recursive_mutex> lock(ev.st->mu);
    if (ev.finished) {
      *done = 1;
      return;
    }
    DeviceScope scope(ev.st->device);
    const cudaError_t q = cudaEventQuery(ev.ev);
    if (q == cudaErrorNotReady) {
      *done = 0;
      return;
    }
    cuda_check(q, "cudaEventQuery");
    ev.finish();
    *done = 1;
  });
}

int ask_b200_event_wait(ask_b200_event* e) {
  return guarded([&] {
    require(e && e->e, "event is NULL");
    EventImpl& ev = *e->e;
    std::lock_guard<std::recursive_mutex> lock(ev.st->mu);
    if (ev.finished) return;
    DeviceScope scope(ev.st->device);
    cuda_check(cudaEventSynchronize(ev.ev), "cudaEventSynchronize");
    ev.finish();
  });
}

int ask_b200_event_release(ask_b200_event* e) {
  delete e;
  return ASK_B200_OK;
}

int ask_b200_allocation_check(const char* allocation_json, int* pass, char* buf, size_t cap, size_t* needed) {
  return guarded([&] {
    require(allocation_json && pass, "argument is NULL");
    const json::Value v = json::Parser(allocation_json).parse();
    check::Verdict verdict;
    if (!v.get("buffer_sizes")) {
      verdict = check::check_plan(parse_check_plan(v));
    } else {
      check::Allocation a;
      a.plan = parse_check_plan(v);
      a.buffer_sizes = index_list(v.at("buffer_sizes"), "buffer_sizes");
      if (const json::Value* as = v.get("assignments"))
        for (const auto& e : as->as_array("assignments")) {
          const auto pair = index_list(e, "assignment");
          require(pair.size() == 2, "an assignment is [buffer, slot]");
          a.assignments.push_back({pair[0], pair[1]});
        }
      if (const json::Value* c = v.get("slot_capacity_bytes")) a.slot_capacity_bytes = index_list(*c, "slot_capacity_bytes");
      if (const json::Value* g = v.get("graph")) a.graph = g->kind == json::Value::Bool && g->b;
      if (const json::Value* d = v.get("dependencies"))
        for (const auto& e : d->as_array("dependencies")) a.dependencies.push_back(index_list(e, "dependencies"));
      verdict = check::check_allocation(a);
    }
    *pass = verdict.pass ? 1 : 0;
    write_text(verdict.explanation, buf, cap, needed);
  });
}

int ask_b200_allocation_assign(const char* plan_json, int graph, char* buf, size_t cap, size_t* needed) {
  return guarded([&] {
    require(plan_json != nullptr, "plan JSON is NULL");
    const json::Value v = json::Parser(plan_json).parse();
    check::Allocation a;
    a.plan = parse_check_plan(v);
    a.buffer_sizes = index_list(v.at("buffer_sizes"), "buffer_sizes");
    require(a.buffer_sizes.size() == a.plan.buffer_count, "allocation buffer sizes differ from the plan");
    const check::Verdict structure = check::check_plan(a.plan);
    require(structure.pass, "plan is invalid: " + structure.explanation);
    if (graph)
      check::assign_graph_slots(a);
    else
      check::assign_stream_slots(a);
    std::ostringstream o;
    o << "{\"assignments\":[";
    for (size_t i = 0; i < a.assignments.size(); ++i)
      o << (i ? "," : "") << "[" << a.assignments[i].buffer << "," << a.assignments[i].slot << "]";
    o << "],\"slot_capacity_bytes\":[";
    for (size_t i = 0; i < a.slot_capacity_bytes.size(); ++i) o << (i ? "," : "") << a.slot_capacity_bytes[i];
    o << "],\"graph\":" << (a.graph ? "true" : "false") << ",\"dependencies\":[";
    for (size_t i = 0; i < a.dependencies.size(); ++i) {
      o << (i ? "," : "") << "[";
      for (size_t j = 0; j < a.dependencies[i].size(); ++j) o << (j ? "," : "") << a.dependencies[i][j];
      o << "]";
    }
    o << "]}";
    write_text(o.str(), buf, cap, needed);
  });
}

}  // extern "C"

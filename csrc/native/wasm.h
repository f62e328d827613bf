// A small WebAssembly interpreter with a WASI preview1 subset, for running RAG
// connectors packaged as `.wasm` command modules: one instantiation per
// request, the request on stdin, the response read back from stdout, with the
// environment and the preopened directories the workspace grants.
//
// Supported: the MVP instruction set plus sign-extension, saturating
// float->int truncation, bulk memory/table operations, multi-value block
// types, reference types (funcref tables).  Not supported: SIMD, threads,
// exceptions, imported memories/tables/globals.  Every memory access is
// bounds-checked, recursion depth and the value stack are capped, and a fuel
// budget plus a wall-clock deadline stop runaway modules; each of these ends
// the run with a Trap instead of harming the host.
//
// Reference counterpart: crates/kapsl-rag/src/runtime/mod.rs:198-331
// (WasmConnectorRuntime on wasmtime with WASI preview1 pipes and preopens).
#pragma once

#include <stdint.h>

#include <chrono>
#include <functional>
#include <map>
#include <stdexcept>
#include <string>
#include <tuple>
#include <unordered_map>
#include <vector>

namespace kapsl {
namespace wasm {

struct Trap : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct LoadError : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct ProcExit {
  int32_t code;
};

enum : uint8_t { I32 = 0x7f, I64 = 0x7e, F32 = 0x7d, F64 = 0x7c, FUNCREF = 0x70, EXTERNREF = 0x6f };

struct FuncType {
  std::vector<uint8_t> params, results;
};

struct Limits {
  uint32_t min = 0;
  uint32_t max = 0xffffffffu;
  bool has_max = false;
};

struct Module {
  struct Import {
    std::string module, name;
    uint32_t type = 0;  // function imports only
  };
  struct Code {
    std::vector<uint8_t> locals;  // declared local types, expanded
    uint32_t begin = 0, end = 0;  // body [begin, end) in `bytes`, end at the final 0x0b + 1
  };
  struct Global {
    uint8_t type = I32;
    bool mut = false;
    uint32_t init = 0;  // offset of the constant expression
  };
  struct Elem {
    uint8_t mode = 0;      // 0 active, 1 passive, 2 declarative
    uint32_t table = 0;
    uint32_t offset = 0;   // constant expression (active)
    std::vector<int64_t> funcs;  // function index or -1 (null)
  };
  struct Data {
    bool active = true;
    uint32_t offset = 0;   // constant expression (active)
    uint32_t begin = 0, len = 0;
  };

  std::vector<uint8_t> bytes;
  std::vector<FuncType> types;
  std::vector<Import> imports;
  std::vector<uint32_t> func_types;  // imported functions first
  uint32_t num_imports = 0;
  std::vector<Code> codes;
  bool has_memory = false;
  Limits memory;
  bool has_table = false;
  Limits table;
  std::vector<Global> globals;
  std::map<std::string, std::pair<uint8_t, uint32_t>> exports;  // name -> (kind, index)
  int64_t start = -1;
  std::vector<Elem> elems;
  std::vector<Data> datas;

  static Module parse(const std::string& bytes);
};

class Instance;
// Host function: args and results in the interpreter's 64-bit slots.
using HostFn = std::function<void(Instance&, const uint64_t* args, uint64_t* results)>;

struct RunLimits {
  uint64_t fuel = 4000000000ull;  // instructions (approximately)
  double timeout_s = 30.0;
  uint32_t max_pages = 16384;     // 1 GiB of linear memory
  uint32_t max_depth = 1024;      // nested calls
  uint32_t max_stack = 1u << 20;  // value-stack slots
};

class Instance {
 public:
  // `host` resolves every function import by (module, name); a missing one is a LoadError.
  Instance(Module m, const std::function<HostFn(const std::string&, const std::string&, const FuncType&)>& host,
           RunLimits lim = {});

  std::vector<uint64_t> invoke(const std::string& export_name, const std::vector<uint64_t>& args);
  std::vector<uint64_t> call(uint32_t func, const std::vector<uint64_t>& args);
  const FuncType& type_of(uint32_t func) const { return mod_.types[mod_.func_types[func]]; }
  uint32_t export_func(const std::string& name) const;

  // Linear memory, bounds-checked for host functions.
  uint8_t* mem(uint64_t addr, uint64_t len);
  uint64_t mem_size() const { return memory_.size(); }

 private:
  struct Ctl {
    uint32_t end = 0, els = 0;  // positions of the matching `end` / `else` opcodes (0: none)
  };
  struct Label {
    uint32_t cont;    // where a branch continues (loop: body start; block/if: after `end`)
    uint32_t height;  // value-stack height below the block's parameters
    uint16_t arity;   // values a branch carries
    uint16_t results; // values left by falling through the `end`
    bool loop;
  };

  void exec(uint32_t func, uint32_t base, uint32_t depth);
  uint64_t const_expr(uint32_t pc) const;
  const std::unordered_map<uint32_t, Ctl>& control(uint32_t defined);
  void block_sig(uint32_t& pc, uint16_t& params, uint16_t& results) const;
  void tick(uint64_t n);

  Module mod_;
  RunLimits lim_;
  std::vector<HostFn> host_;
  std::vector<uint8_t> memory_;
  uint32_t mem_max_pages_ = 0;
  std::vector<int64_t> table_;  // function index or -1
  uint32_t table_max_ = 0;
  std::vector<uint64_t> globals_;
  std::vector<uint8_t> data_dropped_, elem_dropped_;
  std::vector<uint64_t> stack_;
  uint32_t sp_ = 0;
  std::vector<std::unordered_map<uint32_t, Ctl>> ctl_;
  std::vector<uint8_t> ctl_done_;
  uint64_t fuel_ = 0;
  std::chrono::steady_clock::time_point deadline_;
};

// WASI preview1 for a command module run once.
struct WasiConfig {
  std::string stdin_data;
  std::vector<std::pair<std::string, std::string>> env;
  std::vector<std::tuple<std::string, std::string, bool>> preopens;  // (host dir, guest path, read only)
  std::vector<std::string> args{"connector"};
  size_t stdout_cap = 4u << 20;
  size_t stderr_cap = 256u << 10;
};

struct WasiResult {
  int32_t exit_code = 0;
  std::string out, err;
};

// Instantiates `module_bytes` with WASI imports and runs its `_start`.
// Throws LoadError (bad module / unknown import) or Trap.
WasiResult run_wasi(const std::string& module_bytes, const WasiConfig& cfg, RunLimits lim = {});

}  // namespace wasm
}  // namespace kapsl

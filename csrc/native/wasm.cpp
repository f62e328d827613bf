// WebAssembly module decoder and interpreter (see wasm.h).  The WASI preview1
// host functions live in wasi.cpp.
#include "wasm.h"

#include <cmath>
#include <cstring>
#include <limits>

namespace kapsl {
namespace wasm {

namespace {

constexpr uint64_t kPage = 65536;
constexpr uint64_t kNullRef = ~0ull;

// Bounds-checked little-endian / LEB128 reader over [p + i, p + n).
struct Rd {
  const uint8_t* p;
  size_t n, i;
  uint8_t u8() {
    if (i >= n) throw LoadError("unexpected end of module");
    return p[i++];
  }
  // at most ceil(bits / 7) bytes, as the binary format allows
  uint64_t leb_u(int bits) {
    uint64_t v = 0;
    for (int shift = 0;; shift += 7) {
      if (shift >= (bits + 6) / 7 * 7) throw LoadError("LEB128 value too long");
      const uint8_t b = u8();
      v |= (uint64_t)(b & 0x7f) << shift;
      if (!(b & 0x80)) break;
    }
    return v;
  }
  int64_t leb_s(int bits) {
    uint64_t v = 0;
    int shift = 0;
    uint8_t b;
    do {
      if (shift >= (bits + 6) / 7 * 7) throw LoadError("LEB128 value too long");
      b = u8();
      v |= (uint64_t)(b & 0x7f) << shift;
      shift += 7;
    } while (b & 0x80);
    if (shift < 64 && (b & 0x40)) v |= ~0ull << shift;
    return (int64_t)v;
  }
  uint32_t u32() {
    const uint64_t v = leb_u(32);
    if (v > 0xffffffffull) throw LoadError("u32 out of range");
    return (uint32_t)v;
  }
  std::string name() {
    const uint32_t len = u32();
    if (len > n - i) throw LoadError("name past the end");
    std::string s(reinterpret_cast<const char*>(p + i), len);
    i += len;
    return s;
  }
  void skip(size_t k) {
    if (k > n - i) throw LoadError("unexpected end of module");
    i += k;
  }
};

bool valtype_ok(uint8_t t) { return t == I32 || t == I64 || t == F32 || t == F64 || t == FUNCREF || t == EXTERNREF; }

Limits read_limits(Rd& r) {
  Limits l;
  const uint8_t flag = r.u8();
  if (flag > 1) throw LoadError("shared or 64-bit limits are not supported");
  l.min = r.u32();
  if (flag == 1) {
    l.max = r.u32();
    l.has_max = true;
    if (l.max < l.min) throw LoadError("limits: max below min");
  }
  return l;
}

// Skips a constant expression (up to and including its `end`); returns its offset.
uint32_t skip_const_expr(Rd& r) {
  const uint32_t at = (uint32_t)r.i;
  for (;;) {
    const uint8_t op = r.u8();
    switch (op) {
      case 0x0b: return at;
      case 0x41: r.leb_s(32); break;
      case 0x42: r.leb_s(64); break;
      case 0x43: r.skip(4); break;
      case 0x44: r.skip(8); break;
      case 0x23: case 0xd2: r.u32(); break;
      case 0xd0: r.u8(); break;
      default: throw LoadError("unsupported instruction in a constant expression");
    }
  }
}

// Reads an element-segment expression (ref.func x / ref.null t).
int64_t read_elem_expr(Rd& r) {
  const uint8_t op = r.u8();
  int64_t v;
  if (op == 0xd2) {
    v = r.u32();
  } else if (op == 0xd0) {
    r.u8();
    v = -1;
  } else {
    throw LoadError("unsupported element expression");
  }
  if (r.u8() != 0x0b) throw LoadError("element expression without end");
  return v;
}

template <class T>
T ld(const uint8_t* p) {
  T v;
  std::memcpy(&v, p, sizeof(T));
  return v;
}
template <class T>
void st(uint8_t* p, T v) {
  std::memcpy(p, &v, sizeof(T));
}

inline float as_f32(uint64_t v) {
  const uint32_t u = (uint32_t)v;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
inline double as_f64(uint64_t v) {
  double d;
  std::memcpy(&d, &v, 8);
  return d;
}
inline uint64_t of_f32(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
}
inline uint64_t of_f64(double d) {
  uint64_t u;
  std::memcpy(&u, &d, 8);
  return u;
}

template <class F>
F fmin_wasm(F a, F b) {
  if (std::isnan(a) || std::isnan(b)) return std::numeric_limits<F>::quiet_NaN();
  if (a == b) return std::signbit(a) ? a : b;  // min(-0, +0) = -0
  return a < b ? a : b;
}
template <class F>
F fmax_wasm(F a, F b) {
  if (std::isnan(a) || std::isnan(b)) return std::numeric_limits<F>::quiet_NaN();
  if (a == b) return std::signbit(a) ? b : a;  // max(-0, +0) = +0
  return a > b ? a : b;
}

[[noreturn]] void trap(const char* what) { throw Trap(what); }

// float -> integer, trapping (checked) or clamping (saturating); x promoted to double
int32_t trunc_i32_s(double x) {
  if (std::isnan(x)) trap("invalid conversion to integer");
  const double t = std::trunc(x);
  if (!(t >= -2147483648.0 && t <= 2147483647.0)) trap("integer overflow");
  return (int32_t)t;
}
uint32_t trunc_i32_u(double x) {
  if (std::isnan(x)) trap("invalid conversion to integer");
  const double t = std::trunc(x);
  if (!(t >= 0.0 && t <= 4294967295.0)) trap("integer overflow");
  return (uint32_t)t;
}
int64_t trunc_i64_s(double x) {
  if (std::isnan(x)) trap("invalid conversion to integer");
  const double t = std::trunc(x);
  if (!(t >= -9223372036854775808.0 && t < 9223372036854775808.0)) trap("integer overflow");
  return (int64_t)t;
}
uint64_t trunc_i64_u(double x) {
  if (std::isnan(x)) trap("invalid conversion to integer");
  const double t = std::trunc(x);
  if (!(t >= 0.0 && t < 18446744073709551616.0)) trap("integer overflow");
  return (uint64_t)t;
}
int32_t sat_i32_s(double x) {
  if (std::isnan(x)) return 0;
  if (x <= -2147483648.0) return std::numeric_limits<int32_t>::min();
  if (x >= 2147483647.0) return std::numeric_limits<int32_t>::max();
  return (int32_t)std::trunc(x);
}
uint32_t sat_i32_u(double x) {
  if (std::isnan(x) || x <= 0.0) return 0;
  if (x >= 4294967295.0) return 0xffffffffu;
  return (uint32_t)std::trunc(x);
}
int64_t sat_i64_s(double x) {
  if (std::isnan(x)) return 0;
  if (x <= -9223372036854775808.0) return std::numeric_limits<int64_t>::min();
  if (x >= 9223372036854775808.0) return std::numeric_limits<int64_t>::max();
  return (int64_t)std::trunc(x);
}
uint64_t sat_i64_u(double x) {
  if (std::isnan(x) || x <= 0.0) return 0;
  if (x >= 18446744073709551616.0) return ~0ull;
  return (uint64_t)std::trunc(x);
}

uint32_t rotl32(uint32_t x, uint32_t k) {
  k &= 31;
  return k ? (x << k) | (x >> (32 - k)) : x;
}
uint32_t rotr32(uint32_t x, uint32_t k) {
  k &= 31;
  return k ? (x >> k) | (x << (32 - k)) : x;
}
uint64_t rotl64(uint64_t x, uint64_t k) {
  k &= 63;
  return k ? (x << k) | (x >> (64 - k)) : x;
}
uint64_t rotr64(uint64_t x, uint64_t k) {
  k &= 63;
  return k ? (x >> k) | (x << (64 - k)) : x;
}

}  // namespace

// ---------------------------------------------------------------- decoder
Module Module::parse(const std::string& src) {
  Module m;
  m.bytes.assign(src.begin(), src.end());
  Rd r{m.bytes.data(), m.bytes.size(), 0};
  if (r.n < 8 || std::memcmp(r.p, "\0asm", 4) != 0) throw LoadError("not a WebAssembly module");
  if (r.p[4] != 1 || r.p[5] || r.p[6] || r.p[7]) throw LoadError("unsupported WebAssembly version");
  r.i = 8;
  std::vector<uint32_t> decl;
  bool have_code = false;
  while (r.i < r.n) {
    const uint8_t id = r.u8();
    const uint32_t size = r.u32();
    if (size > r.n - r.i) throw LoadError("section past the end of the module");
    Rd s{r.p, r.i + size, r.i};
    switch (id) {
      case 0:  // custom
        s.i = s.n;
        break;
      case 1: {
        const uint32_t n = s.u32();
        for (uint32_t k = 0; k < n; ++k) {
          if (s.u8() != 0x60) throw LoadError("malformed function type");
          FuncType t;
          for (uint32_t c = s.u32(), j = 0; j < c; ++j) t.params.push_back(s.u8());
          for (uint32_t c = s.u32(), j = 0; j < c; ++j) t.results.push_back(s.u8());
          for (uint8_t v : t.params) if (!valtype_ok(v)) throw LoadError("bad value type");
          for (uint8_t v : t.results) if (!valtype_ok(v)) throw LoadError("bad value type");
          if (t.results.size() > 16) throw LoadError("more than 16 results");
          m.types.push_back(std::move(t));
        }
        break;
      }
      case 2: {
        const uint32_t n = s.u32();
        for (uint32_t k = 0; k < n; ++k) {
          Import im;
          im.module = s.name();
          im.name = s.name();
          const uint8_t kind = s.u8();
          if (kind != 0) throw LoadError("only function imports are supported (" + im.module + "." + im.name + ")");
          im.type = s.u32();
          if (im.type >= m.types.size()) throw LoadError("import type index out of range");
          m.imports.push_back(im);
          m.func_types.push_back(im.type);
        }
        m.num_imports = (uint32_t)m.imports.size();
        break;
      }
      case 3: {
        const uint32_t n = s.u32();
        for (uint32_t k = 0; k < n; ++k) {
          const uint32_t t = s.u32();
          if (t >= m.types.size()) throw LoadError("function type index out of range");
          decl.push_back(t);
        }
        break;
      }
      case 4: {
        const uint32_t n = s.u32();
        if (n > 1) throw LoadError("more than one table");
        if (n == 1) {
          if (s.u8() != FUNCREF) throw LoadError("only funcref tables are supported");
          m.table = read_limits(s);
          m.has_table = true;
        }
        break;
      }
      case 5: {
        const uint32_t n = s.u32();
        if (n > 1) throw LoadError("more than one memory");
        if (n == 1) {
          m.memory = read_limits(s);
          m.has_memory = true;
          if (m.memory.min > 65536 || (m.memory.has_max && m.memory.max > 65536))
            throw LoadError("memory limits above 4 GiB");
        }
        break;
      }
      case 6: {
        const uint32_t n = s.u32();
        for (uint32_t k = 0; k < n; ++k) {
          Global g;
          g.type = s.u8();
          if (!valtype_ok(g.type)) throw LoadError("bad global type");
          const uint8_t mut = s.u8();
          if (mut > 1) throw LoadError("bad global mutability");
          g.mut = mut == 1;
          g.init = skip_const_expr(s);
          m.globals.push_back(g);
        }
        break;
      }
      case 7: {
        const uint32_t n = s.u32();
        for (uint32_t k = 0; k < n; ++k) {
          std::string nm = s.name();
          const uint8_t kind = s.u8();
          const uint32_t idx = s.u32();
          m.exports[nm] = {kind, idx};
        }
        break;
      }
      case 8:
        m.start = s.u32();
        break;
      case 9: {
        const uint32_t n = s.u32();
        for (uint32_t k = 0; k < n; ++k) {
          Elem e;
          const uint32_t flags = s.u32();
          if (flags > 7) throw LoadError("bad element segment flags");
          const bool exprs = flags & 4;
          if (flags & 1) {
            e.mode = (flags & 2) ? 2 : 1;
          } else {
            e.mode = 0;
            if (flags & 2) e.table = s.u32();
            e.offset = skip_const_expr(s);
          }
          if (flags & 3) {  // element kind / reference type present
            const uint8_t kind = s.u8();
            if (exprs ? kind != FUNCREF : kind != 0x00) throw LoadError("only funcref element segments");
          }
          const uint32_t cnt = s.u32();
          for (uint32_t j = 0; j < cnt; ++j) e.funcs.push_back(exprs ? read_elem_expr(s) : (int64_t)s.u32());
          m.elems.push_back(std::move(e));
        }
        break;
      }
      case 10: {
        const uint32_t n = s.u32();
        if (n != decl.size()) throw LoadError("function and code section counts differ");
        for (uint32_t k = 0; k < n; ++k) {
          const uint32_t size2 = s.u32();
          if (size2 > s.n - s.i) throw LoadError("function body past the end");
          Rd b{s.p, s.i + size2, s.i};
          Code c;
          uint64_t total = 0;
          for (uint32_t groups = b.u32(), j = 0; j < groups; ++j) {
            const uint32_t cnt = b.u32();
            const uint8_t t = b.u8();
            if (!valtype_ok(t)) throw LoadError("bad local type");
            total += cnt;
            if (total > 50000) throw LoadError("too many locals");
            c.locals.insert(c.locals.end(), cnt, t);
          }
          c.begin = (uint32_t)b.i;
          c.end = (uint32_t)b.n;
          if (c.end <= c.begin || m.bytes[c.end - 1] != 0x0b) throw LoadError("function body without end");
          m.codes.push_back(std::move(c));
          s.i = b.n;
        }
        have_code = true;
        break;
      }
      case 11: {
        const uint32_t n = s.u32();
        for (uint32_t k = 0; k < n; ++k) {
          Data d;
          const uint32_t flags = s.u32();
          if (flags == 1) {
            d.active = false;
          } else if (flags == 0 || flags == 2) {
            if (flags == 2 && s.u32() != 0) throw LoadError("data segment for a memory other than 0");
            d.offset = skip_const_expr(s);
          } else {
            throw LoadError("bad data segment flags");
          }
          d.len = s.u32();
          if (d.len > s.n - s.i) throw LoadError("data segment past the end");
          d.begin = (uint32_t)s.i;
          s.i += d.len;
          m.datas.push_back(d);
        }
        break;
      }
      case 12:
        s.u32();
        break;
      default:
        throw LoadError("unknown section " + std::to_string(id));
    }
    if (s.i != s.n) throw LoadError("section size mismatch (section " + std::to_string(id) + ")");
    r.i = s.n;
  }
  if (!decl.empty() && !have_code) throw LoadError("functions without a code section");
  for (uint32_t t : decl) m.func_types.push_back(t);
  const uint64_t nf = m.func_types.size();
  for (auto& [nm, ex] : m.exports) {
    if (ex.first == 0 && ex.second >= nf) throw LoadError("export of a missing function: " + nm);
    if (ex.first == 2 && (!m.has_memory || ex.second != 0)) throw LoadError("export of a missing memory: " + nm);
  }
  if (m.start >= (int64_t)nf) throw LoadError("start function out of range");
  for (auto& e : m.elems)
    for (int64_t f : e.funcs)
      if (f >= (int64_t)nf) throw LoadError("element refers to a missing function");
  return m;
}

// --------------------------------------------------------------- instance
Instance::Instance(Module m,
                   const std::function<HostFn(const std::string&, const std::string&, const FuncType&)>& host,
                   RunLimits lim)
    : mod_(std::move(m)), lim_(lim) {
  fuel_ = lim_.fuel;
  deadline_ = std::chrono::steady_clock::now() +
              std::chrono::duration_cast<std::chrono::steady_clock::duration>(std::chrono::duration<double>(lim_.timeout_s));
  for (auto& im : mod_.imports) {
    HostFn fn = host(im.module, im.name, mod_.types[im.type]);
    if (!fn) throw LoadError("unknown import " + im.module + "." + im.name);
    host_.push_back(std::move(fn));
  }
  if (mod_.has_memory) {
    if (mod_.memory.min > lim_.max_pages) throw LoadError("initial memory above the configured cap");
    memory_.assign((size_t)mod_.memory.min * kPage, 0);
    mem_max_pages_ = std::min<uint32_t>(mod_.memory.has_max ? mod_.memory.max : 65536, lim_.max_pages);
  }
  if (mod_.has_table) {
    if (mod_.table.min > (1u << 20)) throw LoadError("table too large");
    table_.assign(mod_.table.min, -1);
    table_max_ = std::min<uint32_t>(mod_.table.has_max ? mod_.table.max : (1u << 20), 1u << 20);
  }
  for (auto& g : mod_.globals) globals_.push_back(const_expr(g.init));
  stack_.assign(lim_.max_stack, 0);
  ctl_.resize(mod_.codes.size());
  ctl_done_.assign(mod_.codes.size(), 0);
  data_dropped_.assign(mod_.datas.size(), 0);
  elem_dropped_.assign(mod_.elems.size(), 0);
  for (size_t k = 0; k < mod_.elems.size(); ++k) {
    const auto& e = mod_.elems[k];
    if (e.mode == 0) {
      if (e.table != 0 || !mod_.has_table) throw LoadError("element segment without a table");
      const uint64_t off = (uint32_t)const_expr(e.offset);
      if (off + e.funcs.size() > table_.size()) throw Trap("out of bounds table access (element segment)");
      for (size_t j = 0; j < e.funcs.size(); ++j) table_[off + j] = e.funcs[j];
    }
    if (e.mode != 1) elem_dropped_[k] = 1;
  }
  for (size_t k = 0; k < mod_.datas.size(); ++k) {
    const auto& d = mod_.datas[k];
    if (!d.active) continue;
    const uint64_t off = (uint32_t)const_expr(d.offset);
    if (off + d.len > memory_.size()) throw Trap("out of bounds memory access (data segment)");
    if (d.len) std::memcpy(memory_.data() + off, mod_.bytes.data() + d.begin, d.len);
    data_dropped_[k] = 1;
  }
  if (mod_.start >= 0) call((uint32_t)mod_.start, {});
}

uint64_t Instance::const_expr(uint32_t pc) const {
  Rd r{mod_.bytes.data(), mod_.bytes.size(), pc};
  uint64_t v = 0;
  const uint8_t op = r.u8();
  switch (op) {
    case 0x41: v = (uint32_t)(int32_t)r.leb_s(32); break;
    case 0x42: v = (uint64_t)r.leb_s(64); break;
    case 0x43: v = ld<uint32_t>(r.p + r.i); r.i += 4; break;
    case 0x44: v = ld<uint64_t>(r.p + r.i); r.i += 8; break;
    case 0x23: {
      const uint32_t g = r.u32();
      if (g >= globals_.size()) throw LoadError("constant expression reads a later global");
      v = globals_[g];
      break;
    }
    case 0xd2: v = r.u32(); break;
    case 0xd0: r.u8(); v = kNullRef; break;
    default: throw LoadError("unsupported constant expression");
  }
  if (r.u8() != 0x0b) throw LoadError("constant expression with more than one instruction");
  return v;
}

uint8_t* Instance::mem(uint64_t addr, uint64_t len) {
  if (addr > memory_.size() || len > memory_.size() - addr) trap("out of bounds memory access");
  return memory_.data() + addr;
}

uint32_t Instance::export_func(const std::string& name) const {
  auto it = mod_.exports.find(name);
  if (it == mod_.exports.end() || it->second.first != 0) throw LoadError("no exported function " + name);
  return it->second.second;
}

std::vector<uint64_t> Instance::invoke(const std::string& name, const std::vector<uint64_t>& args) {
  return call(export_func(name), args);
}

std::vector<uint64_t> Instance::call(uint32_t f, const std::vector<uint64_t>& args) {
  if (f >= mod_.func_types.size()) throw Trap("function index out of range");
  const FuncType& t = type_of(f);
  if (args.size() != t.params.size()) throw Trap("wrong number of arguments");
  const uint32_t base = sp_;
  if ((uint64_t)base + args.size() + 16 > stack_.size()) trap("value stack exhausted");
  for (uint64_t a : args) stack_[sp_++] = a;
  if (f < mod_.num_imports) {
    uint64_t res[16] = {};
    host_[f](*this, stack_.data() + base, res);
    sp_ = base;
    return std::vector<uint64_t>(res, res + t.results.size());
  }
  exec(f, base, 1);
  std::vector<uint64_t> out(stack_.begin() + base, stack_.begin() + base + t.results.size());
  sp_ = base;
  return out;
}

void Instance::tick(uint64_t n) {
  if (fuel_ <= n) trap("fuel exhausted");
  fuel_ -= n;
  if (std::chrono::steady_clock::now() > deadline_) trap("deadline exceeded");
}

void Instance::block_sig(uint32_t& pc, uint16_t& params, uint16_t& results) const {
  Rd r{mod_.bytes.data(), mod_.bytes.size(), pc};
  const int64_t bt = r.leb_s(33);
  pc = (uint32_t)r.i;
  if (bt == -64) {
    params = results = 0;
  } else if (bt < 0) {
    params = 0;
    results = 1;
  } else {
    if ((uint64_t)bt >= mod_.types.size()) throw Trap("block type index out of range");
    params = (uint16_t)mod_.types[bt].params.size();
    results = (uint16_t)mod_.types[bt].results.size();
  }
}

// Matching end/else of every block of a function, found by decoding the body
// once; decoding also checks that every immediate lies inside the body.
const std::unordered_map<uint32_t, Instance::Ctl>& Instance::control(uint32_t k) {
  if (ctl_done_[k]) return ctl_[k];
  const auto& c = mod_.codes[k];
  Rd r{mod_.bytes.data(), c.end, c.begin};
  auto& map = ctl_[k];
  std::vector<uint32_t> open;
  bool closed = false;  // the function's own `end` (the last byte) was reached with no block open
  while (r.i < r.n) {
    const uint32_t at = (uint32_t)r.i;
    const uint8_t op = r.u8();
    switch (op) {
      case 0x02: case 0x03: case 0x04:
        r.leb_s(33);
        open.push_back(at);
        map[at] = Ctl{};
        break;
      case 0x05:
        if (open.empty() || mod_.bytes[open.back()] != 0x04 || map[open.back()].els)
          throw LoadError("else without a matching if");
        map[open.back()].els = at;
        break;
      case 0x0b:
        if (open.empty()) {
          if (r.i != r.n) throw LoadError("end of the function before the end of its body");
          closed = true;
        } else {
          map[open.back()].end = at;
          open.pop_back();
        }
        break;
      case 0x0c: case 0x0d: case 0x10: case 0x20: case 0x21: case 0x22: case 0x23: case 0x24: case 0x25:
      case 0x26: case 0xd2:
        r.u32();
        break;
      case 0x0e:
        for (uint32_t n = r.u32(), j = 0; j <= n; ++j) r.u32();
        break;
      case 0x11:
        r.u32();
        r.u32();
        break;
      case 0x1c:
        for (uint32_t n = r.u32(), j = 0; j < n; ++j) r.u8();
        break;
      case 0x3f: case 0x40: case 0xd0:
        r.u8();
        break;
      case 0x41: r.leb_s(32); break;
      case 0x42: r.leb_s(64); break;
      case 0x43: r.skip(4); break;
      case 0x44: r.skip(8); break;
      case 0xfc: {
        const uint32_t sub = r.u32();
        if (sub <= 7) break;
        if (sub == 8) { r.u32(); r.u8(); break; }
        if (sub == 9 || sub == 13 || (sub >= 15 && sub <= 17)) { r.u32(); break; }
        if (sub == 10) { r.u8(); r.u8(); break; }
        if (sub == 11) { r.u8(); break; }
        if (sub == 12 || sub == 14) { r.u32(); r.u32(); break; }
        throw LoadError("unsupported 0xfc instruction " + std::to_string(sub));
      }
      default:
        if (op >= 0x28 && op <= 0x3e) {  // memarg
          r.u32();
          r.u32();
        } else if (op == 0x00 || op == 0x01 || op == 0x0f || op == 0x1a || op == 0x1b || op == 0xd1 ||
                   (op >= 0x45 && op <= 0xc4)) {
          // no immediates
        } else {
          throw LoadError("unsupported instruction 0x" + std::to_string(op));
        }
    }
  }
  if (!open.empty() || !closed) throw LoadError("unterminated block");
  ctl_done_[k] = 1;
  return map;
}

// ------------------------------------------------------------ interpreter
void Instance::exec(uint32_t f, uint32_t base, uint32_t depth) {
  if (depth > lim_.max_depth) trap("call stack exhausted");
  const uint32_t k = f - mod_.num_imports;
  const auto& code = mod_.codes[k];
  const auto& ctl = control(k);
  const FuncType& ft = type_of(f);
  const uint32_t nparams = (uint32_t)ft.params.size();
  const uint32_t nlocals = nparams + (uint32_t)code.locals.size();
  const uint16_t nres = (uint16_t)ft.results.size();
  uint64_t* S = stack_.data();
  const uint32_t cap = (uint32_t)stack_.size();
  uint32_t sp = base + nparams;
  if ((uint64_t)base + nlocals + 64 > cap) trap("value stack exhausted");
  for (uint32_t j = nparams; j < nlocals; ++j) S[sp++] = 0;
  const uint32_t lbase = base + nlocals;
  const uint8_t* B = mod_.bytes.data();
  uint32_t pc = code.begin;
  std::vector<Label> labels;
  labels.reserve(16);
  labels.push_back(Label{code.end - 1, lbase, nres, nres, false});
  uint64_t budget = 0;

  auto u32 = [&]() -> uint32_t {
    uint32_t v = 0;
    for (int shift = 0;; shift += 7) {
      const uint8_t b = B[pc++];
      v |= (uint32_t)(b & 0x7f) << shift;
      if (!(b & 0x80)) return v;
    }
  };
  // immediates were bounds- and length-checked when the body was decoded (control())
  auto s64 = [&]() -> int64_t {
    uint64_t v = 0;
    int shift = 0;
    uint8_t b;
    do {
      b = B[pc++];
      v |= (uint64_t)(b & 0x7f) << shift;
      shift += 7;
    } while (b & 0x80);
    if (shift < 64 && (b & 0x40)) v |= ~0ull << shift;
    return (int64_t)v;
  };
#define NEED(n)                                         \
  do {                                                  \
    if (sp < lbase + (uint32_t)(n)) trap("value stack underflow"); \
  } while (0)
#define PUSH(v)                                          \
  do {                                                   \
    if (sp >= cap) trap("value stack exhausted");        \
    S[sp++] = (v);                                       \
  } while (0)
#define TOP S[sp - 1]
#define BIN32(expr)                                     \
  do {                                                  \
    NEED(2);                                            \
    const uint32_t b = (uint32_t)S[sp - 1], a = (uint32_t)S[sp - 2]; \
    (void)a; (void)b;                                   \
    --sp;                                               \
    S[sp - 1] = (uint32_t)(expr);                       \
  } while (0)
#define BIN64(expr)                                     \
  do {                                                  \
    NEED(2);                                            \
    const uint64_t b = S[sp - 1], a = S[sp - 2];        \
    (void)a; (void)b;                                   \
    --sp;                                               \
    S[sp - 1] = (uint64_t)(expr);                       \
  } while (0)
#define CMP32(expr) BIN32((expr) ? 1u : 0u)
#define CMP64(expr)                                     \
  do {                                                  \
    NEED(2);                                            \
    const uint64_t b = S[sp - 1], a = S[sp - 2];        \
    (void)a; (void)b;                                   \
    --sp;                                               \
    S[sp - 1] = (expr) ? 1u : 0u;                       \
  } while (0)
#define FBIN32(expr)                                    \
  do {                                                  \
    NEED(2);                                            \
    const float b = as_f32(S[sp - 1]), a = as_f32(S[sp - 2]); \
    --sp;                                               \
    S[sp - 1] = of_f32(expr);                           \
  } while (0)
#define FBIN64(expr)                                    \
  do {                                                  \
    NEED(2);                                            \
    const double b = as_f64(S[sp - 1]), a = as_f64(S[sp - 2]); \
    --sp;                                               \
    S[sp - 1] = of_f64(expr);                           \
  } while (0)
#define FCMP32(expr)                                    \
  do {                                                  \
    NEED(2);                                            \
    const float b = as_f32(S[sp - 1]), a = as_f32(S[sp - 2]); \
    --sp;                                               \
    S[sp - 1] = (expr) ? 1u : 0u;                       \
  } while (0)
#define FCMP64(expr)                                    \
  do {                                                  \
    NEED(2);                                            \
    const double b = as_f64(S[sp - 1]), a = as_f64(S[sp - 2]); \
    --sp;                                               \
    S[sp - 1] = (expr) ? 1u : 0u;                       \
  } while (0)
#define UN(expr)                                        \
  do {                                                  \
    NEED(1);                                            \
    const uint64_t a = S[sp - 1];                       \
    (void)a;                                            \
    S[sp - 1] = (expr);                                 \
  } while (0)

  // effective address of a load/store of `size` bytes (pops the base address)
  auto addr = [&](uint32_t size) -> uint8_t* {
    u32();  // alignment hint
    const uint64_t off = u32();
    NEED(1);
    const uint64_t ea = (uint64_t)(uint32_t)S[--sp] + off;
    if (ea + size > memory_.size()) trap("out of bounds memory access");
    return memory_.data() + ea;
  };

  // branch to label `depth`; returns true when the branch leaves the function
  auto branch = [&](uint32_t d) -> bool {
    if (d >= labels.size()) trap("branch depth out of range");
    const size_t li = labels.size() - 1 - d;
    const Label L = labels[li];
    NEED(0);
    if (sp < L.height + L.arity) trap("value stack underflow");
    if (sp != L.height + L.arity) {
      std::memmove(S + L.height, S + sp - L.arity, L.arity * sizeof(uint64_t));
      sp = L.height + L.arity;
    }
    if (li == 0) return true;
    if (L.loop) {
      labels.resize(li + 1);
    } else {
      labels.resize(li);
    }
    pc = L.cont;
    return false;
  };

  auto do_call = [&](uint32_t callee) {
    if (callee >= mod_.func_types.size()) trap("call to a missing function");
    const FuncType& t = type_of(callee);
    const uint32_t np = (uint32_t)t.params.size();
    NEED(np);
    if (callee < mod_.num_imports) {
      uint64_t res[16] = {};
      sp_ = sp;
      host_[callee](*this, S + sp - np, res);
      sp -= np;
      for (size_t j = 0; j < t.results.size(); ++j) PUSH(res[j]);
    } else {
      sp_ = sp;
      exec(callee, sp - np, depth + 1);
      sp = sp_;
    }
  };

  for (;;) {
    if (++budget == 4096) {
      tick(budget);
      budget = 0;
    }
    const uint32_t at = pc;
    if (pc >= code.end) trap("execution ran past the end of the function body");
    const uint8_t op = B[pc++];
    switch (op) {
      case 0x00: trap("unreachable executed");
      case 0x01: break;
      case 0x02: case 0x03: {  // block, loop
        uint16_t np, nr;
        block_sig(pc, np, nr);
        NEED(np);
        const auto ci = ctl.find(at);
        if (ci == ctl.end()) trap("block outside the decoded body");
        const Ctl& c = ci->second;
        if (op == 0x02)
          labels.push_back(Label{c.end + 1, sp - np, nr, nr, false});
        else
          labels.push_back(Label{pc, sp - np, np, nr, true});
        break;
      }
      case 0x04: {  // if
        uint16_t np, nr;
        block_sig(pc, np, nr);
        NEED(np + 1);
        const uint32_t cond = (uint32_t)S[--sp];
        const auto ci = ctl.find(at);
        if (ci == ctl.end()) trap("block outside the decoded body");
        const Ctl& c = ci->second;
        if (cond) {
          labels.push_back(Label{c.end + 1, sp - np, nr, nr, false});
        } else if (c.els) {
          labels.push_back(Label{c.end + 1, sp - np, nr, nr, false});
          pc = c.els + 1;
        } else {
          pc = c.end + 1;  // no else: the parameters pass through as results
        }
        break;
      }
      case 0x05: {  // end of a then-branch: continue after the if
        if (labels.size() < 2) trap("else outside a block");
        pc = labels.back().cont;
        labels.pop_back();
        break;
      }
      case 0x0b:
        if (labels.size() == 1) {  // the function's own end
          if (branch(0)) goto done;
        } else {
          labels.pop_back();
        }
        break;
      case 0x0c:
        if (branch(u32())) goto done;
        break;
      case 0x0d: {
        const uint32_t d = u32();
        NEED(1);
        if ((uint32_t)S[--sp] && branch(d)) goto done;
        break;
      }
      case 0x0e: {
        const uint32_t n = u32();
        NEED(1);
        const uint32_t i = (uint32_t)S[--sp];
        uint32_t target = 0;
        for (uint32_t j = 0; j <= n; ++j) {
          const uint32_t d = u32();
          if (j == std::min(i, n)) target = d;
        }
        if (branch(target)) goto done;
        break;
      }
      case 0x0f:
        if (branch((uint32_t)labels.size() - 1)) goto done;
        break;
      case 0x10:
        do_call(u32());
        break;
      case 0x11: {
        const uint32_t ti = u32();
        const uint32_t tab = u32();
        if (tab != 0 || ti >= mod_.types.size()) trap("call_indirect: bad table or type");
        NEED(1);
        const uint32_t i = (uint32_t)S[--sp];
        if (i >= table_.size()) trap("undefined element");
        const int64_t fi = table_[i];
        if (fi < 0) trap("uninitialized element");
        if ((uint64_t)fi >= mod_.func_types.size()) trap("bad function reference");
        const FuncType& want = mod_.types[ti];
        const FuncType& got = type_of((uint32_t)fi);
        if (want.params != got.params || want.results != got.results) trap("indirect call type mismatch");
        do_call((uint32_t)fi);
        break;
      }
      case 0x1a:
        NEED(1);
        --sp;
        break;
      case 0x1b: case 0x1c: {
        if (op == 0x1c)
          for (uint32_t n = u32(), j = 0; j < n; ++j) ++pc;
        NEED(3);
        const uint32_t c = (uint32_t)S[--sp];
        --sp;
        if (!c) S[sp - 1] = S[sp];
        break;
      }
      case 0x20: {
        const uint32_t i = u32();
        if (i >= nlocals) trap("local index out of range");
        PUSH(S[base + i]);
        break;
      }
      case 0x21: {
        const uint32_t i = u32();
        if (i >= nlocals) trap("local index out of range");
        NEED(1);
        S[base + i] = S[--sp];
        break;
      }
      case 0x22: {
        const uint32_t i = u32();
        if (i >= nlocals) trap("local index out of range");
        NEED(1);
        S[base + i] = S[sp - 1];
        break;
      }
      case 0x23: {
        const uint32_t g = u32();
        if (g >= globals_.size()) trap("global index out of range");
        PUSH(globals_[g]);
        break;
      }
      case 0x24: {
        const uint32_t g = u32();
        if (g >= globals_.size() || !mod_.globals[g].mut) trap("global.set of a missing or immutable global");
        NEED(1);
        globals_[g] = S[--sp];
        break;
      }
      case 0x25: {
        if (u32() != 0) trap("table index out of range");
        NEED(1);
        const uint32_t i = (uint32_t)S[sp - 1];
        if (i >= table_.size()) trap("out of bounds table access");
        S[sp - 1] = (uint64_t)table_[i];
        break;
      }
      case 0x26: {
        if (u32() != 0) trap("table index out of range");
        NEED(2);
        const uint64_t v = S[--sp];
        const uint32_t i = (uint32_t)S[--sp];
        if (i >= table_.size()) trap("out of bounds table access");
        if (v != kNullRef && v >= mod_.func_types.size()) trap("bad function reference");
        table_[i] = v == kNullRef ? -1 : (int64_t)v;
        break;
      }
      // loads: the address is popped by addr(), the value pushed
      case 0x28: { const uint8_t* p = addr(4); PUSH(ld<uint32_t>(p)); break; }
      case 0x29: { const uint8_t* p = addr(8); PUSH(ld<uint64_t>(p)); break; }
      case 0x2a: { const uint8_t* p = addr(4); PUSH(ld<uint32_t>(p)); break; }
      case 0x2b: { const uint8_t* p = addr(8); PUSH(ld<uint64_t>(p)); break; }
      case 0x2c: { const uint8_t* p = addr(1); PUSH((uint32_t)(int32_t)ld<int8_t>(p)); break; }
      case 0x2d: { const uint8_t* p = addr(1); PUSH((uint32_t)ld<uint8_t>(p)); break; }
      case 0x2e: { const uint8_t* p = addr(2); PUSH((uint32_t)(int32_t)ld<int16_t>(p)); break; }
      case 0x2f: { const uint8_t* p = addr(2); PUSH((uint32_t)ld<uint16_t>(p)); break; }
      case 0x30: { const uint8_t* p = addr(1); PUSH((uint64_t)(int64_t)ld<int8_t>(p)); break; }
      case 0x31: { const uint8_t* p = addr(1); PUSH((uint64_t)ld<uint8_t>(p)); break; }
      case 0x32: { const uint8_t* p = addr(2); PUSH((uint64_t)(int64_t)ld<int16_t>(p)); break; }
      case 0x33: { const uint8_t* p = addr(2); PUSH((uint64_t)ld<uint16_t>(p)); break; }
      case 0x34: { const uint8_t* p = addr(4); PUSH((uint64_t)(int64_t)ld<int32_t>(p)); break; }
      case 0x35: { const uint8_t* p = addr(4); PUSH((uint64_t)ld<uint32_t>(p)); break; }
      // stores: value on top, address below it
      case 0x36: case 0x37: case 0x38: case 0x39: case 0x3a: case 0x3b: case 0x3c: case 0x3d: case 0x3e: {
        NEED(2);
        const uint64_t v = S[--sp];
        static const uint8_t widths[] = {4, 8, 4, 8, 1, 2, 1, 2, 4};
        const uint32_t w = widths[op - 0x36];
        uint8_t* p = addr(w);
        std::memcpy(p, &v, w);  // little-endian host: the low bytes
        break;
      }
      case 0x3f:
        ++pc;
        PUSH((uint32_t)(memory_.size() / kPage));
        break;
      case 0x40: {
        ++pc;
        NEED(1);
        const uint32_t delta = (uint32_t)S[sp - 1];
        const uint64_t old = memory_.size() / kPage;
        if (!mod_.has_memory || old + delta > mem_max_pages_) {
          S[sp - 1] = 0xffffffffu;
        } else {
          memory_.resize((old + delta) * kPage, 0);
          S[sp - 1] = (uint32_t)old;
        }
        break;
      }
      case 0x41: PUSH((uint32_t)(int32_t)s64()); break;
      case 0x42: PUSH((uint64_t)s64()); break;
      case 0x43: PUSH(ld<uint32_t>(B + pc)); pc += 4; break;
      case 0x44: PUSH(ld<uint64_t>(B + pc)); pc += 8; break;

      case 0x45: UN((uint32_t)a == 0 ? 1u : 0u); break;
      case 0x46: CMP32(a == b); break;
      case 0x47: CMP32(a != b); break;
      case 0x48: CMP32((int32_t)a < (int32_t)b); break;
      case 0x49: CMP32(a < b); break;
      case 0x4a: CMP32((int32_t)a > (int32_t)b); break;
      case 0x4b: CMP32(a > b); break;
      case 0x4c: CMP32((int32_t)a <= (int32_t)b); break;
      case 0x4d: CMP32(a <= b); break;
      case 0x4e: CMP32((int32_t)a >= (int32_t)b); break;
      case 0x4f: CMP32(a >= b); break;
      case 0x50: UN(a == 0 ? 1u : 0u); break;
      case 0x51: CMP64(a == b); break;
      case 0x52: CMP64(a != b); break;
      case 0x53: CMP64((int64_t)a < (int64_t)b); break;
      case 0x54: CMP64(a < b); break;
      case 0x55: CMP64((int64_t)a > (int64_t)b); break;
      case 0x56: CMP64(a > b); break;
      case 0x57: CMP64((int64_t)a <= (int64_t)b); break;
      case 0x58: CMP64(a <= b); break;
      case 0x59: CMP64((int64_t)a >= (int64_t)b); break;
      case 0x5a: CMP64(a >= b); break;
      case 0x5b: FCMP32(a == b); break;
      case 0x5c: FCMP32(a != b); break;
      case 0x5d: FCMP32(a < b); break;
      case 0x5e: FCMP32(a > b); break;
      case 0x5f: FCMP32(a <= b); break;
      case 0x60: FCMP32(a >= b); break;
      case 0x61: FCMP64(a == b); break;
      case 0x62: FCMP64(a != b); break;
      case 0x63: FCMP64(a < b); break;
      case 0x64: FCMP64(a > b); break;
      case 0x65: FCMP64(a <= b); break;
      case 0x66: FCMP64(a >= b); break;

      case 0x67: UN((uint32_t)a ? (uint32_t)__builtin_clz((uint32_t)a) : 32u); break;
      case 0x68: UN((uint32_t)a ? (uint32_t)__builtin_ctz((uint32_t)a) : 32u); break;
      case 0x69: UN((uint32_t)__builtin_popcount((uint32_t)a)); break;
      case 0x6a: BIN32(a + b); break;
      case 0x6b: BIN32(a - b); break;
      case 0x6c: BIN32(a * b); break;
      case 0x6d: {
        NEED(2);
        const int32_t b = (int32_t)S[sp - 1], a = (int32_t)S[sp - 2];
        if (b == 0) trap("integer divide by zero");
        if (a == std::numeric_limits<int32_t>::min() && b == -1) trap("integer overflow");
        --sp;
        S[sp - 1] = (uint32_t)(a / b);
        break;
      }
      case 0x6e: {
        NEED(2);
        const uint32_t b = (uint32_t)S[sp - 1], a = (uint32_t)S[sp - 2];
        if (b == 0) trap("integer divide by zero");
        --sp;
        S[sp - 1] = a / b;
        break;
      }
      case 0x6f: {
        NEED(2);
        const int32_t b = (int32_t)S[sp - 1], a = (int32_t)S[sp - 2];
        if (b == 0) trap("integer divide by zero");
        --sp;
        S[sp - 1] = (uint32_t)(b == -1 ? 0 : a % b);
        break;
      }
      case 0x70: {
        NEED(2);
        const uint32_t b = (uint32_t)S[sp - 1], a = (uint32_t)S[sp - 2];
        if (b == 0) trap("integer divide by zero");
        --sp;
        S[sp - 1] = a % b;
        break;
      }
      case 0x71: BIN32(a & b); break;
      case 0x72: BIN32(a | b); break;
      case 0x73: BIN32(a ^ b); break;
      case 0x74: BIN32(a << (b & 31)); break;
      case 0x75: BIN32((uint32_t)((int32_t)a >> (b & 31))); break;
      case 0x76: BIN32(a >> (b & 31)); break;
      case 0x77: BIN32(rotl32(a, b)); break;
      case 0x78: BIN32(rotr32(a, b)); break;

      case 0x79: UN(a ? (uint64_t)__builtin_clzll(a) : 64u); break;
      case 0x7a: UN(a ? (uint64_t)__builtin_ctzll(a) : 64u); break;
      case 0x7b: UN((uint64_t)__builtin_popcountll(a)); break;
      case 0x7c: BIN64(a + b); break;
      case 0x7d: BIN64(a - b); break;
      case 0x7e: BIN64(a * b); break;
      case 0x7f: {
        NEED(2);
        const int64_t b = (int64_t)S[sp - 1], a = (int64_t)S[sp - 2];
        if (b == 0) trap("integer divide by zero");
        if (a == std::numeric_limits<int64_t>::min() && b == -1) trap("integer overflow");
        --sp;
        S[sp - 1] = (uint64_t)(a / b);
        break;
      }
      case 0x80: {
        NEED(2);
        const uint64_t b = S[sp - 1], a = S[sp - 2];
        if (b == 0) trap("integer divide by zero");
        --sp;
        S[sp - 1] = a / b;
        break;
      }
      case 0x81: {
        NEED(2);
        const int64_t b = (int64_t)S[sp - 1], a = (int64_t)S[sp - 2];
        if (b == 0) trap("integer divide by zero");
        --sp;
        S[sp - 1] = (uint64_t)(b == -1 ? 0 : a % b);
        break;
      }
      case 0x82: {
        NEED(2);
        const uint64_t b = S[sp - 1], a = S[sp - 2];
        if (b == 0) trap("integer divide by zero");
        --sp;
        S[sp - 1] = a % b;
        break;
      }
      case 0x83: BIN64(a & b); break;
      case 0x84: BIN64(a | b); break;
      case 0x85: BIN64(a ^ b); break;
      case 0x86: BIN64(a << (b & 63)); break;
      case 0x87: BIN64((uint64_t)((int64_t)a >> (b & 63))); break;
      case 0x88: BIN64(a >> (b & 63)); break;
      case 0x89: BIN64(rotl64(a, b)); break;
      case 0x8a: BIN64(rotr64(a, b)); break;

      case 0x8b: UN((uint32_t)a & 0x7fffffffu); break;
      case 0x8c: UN((uint32_t)a ^ 0x80000000u); break;
      case 0x8d: UN(of_f32(std::ceil(as_f32(a)))); break;
      case 0x8e: UN(of_f32(std::floor(as_f32(a)))); break;
      case 0x8f: UN(of_f32(std::trunc(as_f32(a)))); break;
      case 0x90: UN(of_f32(std::nearbyint(as_f32(a)))); break;
      case 0x91: UN(of_f32(std::sqrt(as_f32(a)))); break;
      case 0x92: FBIN32(a + b); break;
      case 0x93: FBIN32(a - b); break;
      case 0x94: FBIN32(a * b); break;
      case 0x95: FBIN32(a / b); break;
      case 0x96: FBIN32(fmin_wasm(a, b)); break;
      case 0x97: FBIN32(fmax_wasm(a, b)); break;
      case 0x98: FBIN32(std::copysign(a, b)); break;
      case 0x99: UN(a & 0x7fffffffffffffffull); break;
      case 0x9a: UN(a ^ 0x8000000000000000ull); break;
      case 0x9b: UN(of_f64(std::ceil(as_f64(a)))); break;
      case 0x9c: UN(of_f64(std::floor(as_f64(a)))); break;
      case 0x9d: UN(of_f64(std::trunc(as_f64(a)))); break;
      case 0x9e: UN(of_f64(std::nearbyint(as_f64(a)))); break;
      case 0x9f: UN(of_f64(std::sqrt(as_f64(a)))); break;
      case 0xa0: FBIN64(a + b); break;
      case 0xa1: FBIN64(a - b); break;
      case 0xa2: FBIN64(a * b); break;
      case 0xa3: FBIN64(a / b); break;
      case 0xa4: FBIN64(fmin_wasm(a, b)); break;
      case 0xa5: FBIN64(fmax_wasm(a, b)); break;
      case 0xa6: FBIN64(std::copysign(a, b)); break;

      case 0xa7: UN((uint32_t)a); break;
      case 0xa8: UN((uint32_t)trunc_i32_s(as_f32(a))); break;
      case 0xa9: UN(trunc_i32_u(as_f32(a))); break;
      case 0xaa: UN((uint32_t)trunc_i32_s(as_f64(a))); break;
      case 0xab: UN(trunc_i32_u(as_f64(a))); break;
      case 0xac: UN((uint64_t)(int64_t)(int32_t)(uint32_t)a); break;
      case 0xad: UN((uint64_t)(uint32_t)a); break;
      case 0xae: UN((uint64_t)trunc_i64_s(as_f32(a))); break;
      case 0xaf: UN(trunc_i64_u(as_f32(a))); break;
      case 0xb0: UN((uint64_t)trunc_i64_s(as_f64(a))); break;
      case 0xb1: UN(trunc_i64_u(as_f64(a))); break;
      case 0xb2: UN(of_f32((float)(int32_t)(uint32_t)a)); break;
      case 0xb3: UN(of_f32((float)(uint32_t)a)); break;
      case 0xb4: UN(of_f32((float)(int64_t)a)); break;
      case 0xb5: UN(of_f32((float)a)); break;
      case 0xb6: UN(of_f32((float)as_f64(a))); break;
      case 0xb7: UN(of_f64((double)(int32_t)(uint32_t)a)); break;
      case 0xb8: UN(of_f64((double)(uint32_t)a)); break;
      case 0xb9: UN(of_f64((double)(int64_t)a)); break;
      case 0xba: UN(of_f64((double)a)); break;
      case 0xbb: UN(of_f64((double)as_f32(a))); break;
      case 0xbc: case 0xbd: case 0xbe: case 0xbf: break;  // reinterpret: same bits
      case 0xc0: UN((uint32_t)(int32_t)(int8_t)(uint8_t)a); break;
      case 0xc1: UN((uint32_t)(int32_t)(int16_t)(uint16_t)a); break;
      case 0xc2: UN((uint64_t)(int64_t)(int8_t)(uint8_t)a); break;
      case 0xc3: UN((uint64_t)(int64_t)(int16_t)(uint16_t)a); break;
      case 0xc4: UN((uint64_t)(int64_t)(int32_t)(uint32_t)a); break;

      case 0xd0: ++pc; PUSH(kNullRef); break;
      case 0xd1: UN(a == kNullRef ? 1u : 0u); break;
      case 0xd2: {
        const uint32_t fi = u32();
        if (fi >= mod_.func_types.size()) trap("ref.func of a missing function");
        PUSH(fi);
        break;
      }

      case 0xfc: {
        const uint32_t sub = u32();
        switch (sub) {
          case 0: UN((uint32_t)sat_i32_s(as_f32(a))); break;
          case 1: UN(sat_i32_u(as_f32(a))); break;
          case 2: UN((uint32_t)sat_i32_s(as_f64(a))); break;
          case 3: UN(sat_i32_u(as_f64(a))); break;
          case 4: UN((uint64_t)sat_i64_s(as_f32(a))); break;
          case 5: UN(sat_i64_u(as_f32(a))); break;
          case 6: UN((uint64_t)sat_i64_s(as_f64(a))); break;
          case 7: UN(sat_i64_u(as_f64(a))); break;
          case 8: {  // memory.init
            const uint32_t seg = u32();
            ++pc;
            NEED(3);
            const uint64_t n = (uint32_t)S[--sp], src = (uint32_t)S[--sp], dst = (uint32_t)S[--sp];
            if (seg >= mod_.datas.size()) trap("data segment index out of range");
            const uint64_t len = data_dropped_[seg] ? 0 : mod_.datas[seg].len;
            if (src + n > len || dst + n > memory_.size()) trap("out of bounds memory access");
            if (n) std::memcpy(memory_.data() + dst, B + mod_.datas[seg].begin + src, n);
            break;
          }
          case 9: {
            const uint32_t seg = u32();
            if (seg >= mod_.datas.size()) trap("data segment index out of range");
            data_dropped_[seg] = 1;
            break;
          }
          case 10: {  // memory.copy
            pc += 2;
            NEED(3);
            const uint64_t n = (uint32_t)S[--sp], src = (uint32_t)S[--sp], dst = (uint32_t)S[--sp];
            if (src + n > memory_.size() || dst + n > memory_.size()) trap("out of bounds memory access");
            if (n) std::memmove(memory_.data() + dst, memory_.data() + src, n);
            break;
          }
          case 11: {  // memory.fill
            ++pc;
            NEED(3);
            const uint64_t n = (uint32_t)S[--sp];
            const uint8_t v = (uint8_t)S[--sp];
            const uint64_t dst = (uint32_t)S[--sp];
            if (dst + n > memory_.size()) trap("out of bounds memory access");
            if (n) std::memset(memory_.data() + dst, v, n);
            break;
          }
          case 12: {  // table.init
            const uint32_t seg = u32();
            if (u32() != 0) trap("table index out of range");
            NEED(3);
            const uint64_t n = (uint32_t)S[--sp], src = (uint32_t)S[--sp], dst = (uint32_t)S[--sp];
            if (seg >= mod_.elems.size()) trap("element segment index out of range");
            const auto& fs = mod_.elems[seg].funcs;
            const uint64_t len = elem_dropped_[seg] ? 0 : fs.size();
            if (src + n > len || dst + n > table_.size()) trap("out of bounds table access");
            for (uint64_t j = 0; j < n; ++j) table_[dst + j] = fs[src + j];
            break;
          }
          case 13: {
            const uint32_t seg = u32();
            if (seg >= mod_.elems.size()) trap("element segment index out of range");
            elem_dropped_[seg] = 1;
            break;
          }
          case 14: {  // table.copy
            if (u32() != 0 || u32() != 0) trap("table index out of range");
            NEED(3);
            const uint64_t n = (uint32_t)S[--sp], src = (uint32_t)S[--sp], dst = (uint32_t)S[--sp];
            if (src + n > table_.size() || dst + n > table_.size()) trap("out of bounds table access");
            if (n) std::memmove(table_.data() + dst, table_.data() + src, n * sizeof(int64_t));
            break;
          }
          case 15: {  // table.grow
            if (u32() != 0) trap("table index out of range");
            NEED(2);
            const uint64_t n = (uint32_t)S[--sp];
            const uint64_t v = S[sp - 1];
            if (v != kNullRef && v >= mod_.func_types.size()) trap("bad function reference");
            const uint64_t old = table_.size();
            if (old + n > table_max_) {
              S[sp - 1] = 0xffffffffu;
            } else {
              table_.resize(old + n, v == kNullRef ? -1 : (int64_t)v);
              S[sp - 1] = (uint32_t)old;
            }
            break;
          }
          case 16:
            if (u32() != 0) trap("table index out of range");
            PUSH((uint32_t)table_.size());
            break;
          case 17: {  // table.fill
            if (u32() != 0) trap("table index out of range");
            NEED(3);
            const uint64_t n = (uint32_t)S[--sp];
            const uint64_t v = S[--sp];
            const uint64_t dst = (uint32_t)S[--sp];
            if (v != kNullRef && v >= mod_.func_types.size()) trap("bad function reference");
            if (dst + n > table_.size()) trap("out of bounds table access");
            for (uint64_t j = 0; j < n; ++j) table_[dst + j] = v == kNullRef ? -1 : (int64_t)v;
            break;
          }
          default:
            trap("unsupported 0xfc instruction");
        }
        break;
      }
      default:
        trap("unsupported instruction");
    }
  }
done:
  // results were moved to the function label's height (= lbase); return them at `base`
  if (nres) std::memmove(S + base, S + lbase, nres * sizeof(uint64_t));
  sp_ = base + nres;
  tick(budget);
#undef NEED
#undef PUSH
#undef TOP
#undef BIN32
#undef BIN64
#undef CMP32
#undef CMP64
#undef FBIN32
#undef FBIN64
#undef FCMP32
#undef FCMP64
#undef UN
}

}  // namespace wasm
}  // namespace kapsl

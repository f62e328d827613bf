// WASI preview1 host functions for the interpreter in wasm.cpp: stdin from a
// buffer, stdout/stderr captured with caps, the environment and arguments,
// clocks and randomness, and files under preopened directories (read-only
// directories refuse every mutation; paths never leave their directory:
// absolute paths and ".." are refused, symlinks are not followed, and the
// resolved parent must lie under the preopen).
//
// Reference counterpart: crates/kapsl-rag/src/runtime/mod.rs:198-331
// (wasmtime_wasi preview1 with MemoryInputPipe / MemoryOutputPipe, preopened
// dirs with DirPerms/FilePerms, env from the workspace config).
#include <dirent.h>
#include <fcntl.h>
#include <limits.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstring>
#include <map>
#include <random>

#include "wasm.h"

namespace kapsl {
namespace wasm {

namespace {

enum : uint32_t {
  W_OK_ = 0,
  W_EACCES = 2,
  W_EBADF = 8,
  W_EEXIST = 20,
  W_EINVAL = 28,
  W_EIO = 29,
  W_EISDIR = 31,
  W_ELOOP = 32,
  W_ENAMETOOLONG = 37,
  W_ENOENT = 44,
  W_ENOSPC = 51,
  W_ENOSYS = 52,
  W_ENOTDIR = 54,
  W_ENOTEMPTY = 55,
  W_EPERM = 63,
  W_ESPIPE = 70,
  W_ENOTCAPABLE = 76,
};

constexpr uint64_t RIGHTS_ALL = (1ull << 29) - 1;
// rights that modify the file system or a file
constexpr uint64_t RIGHTS_MUTATE = (1ull << 0) | (1ull << 3) | (1ull << 4) | (1ull << 6) | (1ull << 8) | (1ull << 9) |
                                   (1ull << 10) | (1ull << 11) | (1ull << 12) | (1ull << 16) | (1ull << 17) |
                                   (1ull << 19) | (1ull << 20) | (1ull << 22) | (1ull << 23) | (1ull << 24) |
                                   (1ull << 25) | (1ull << 26);
constexpr uint64_t RIGHT_FD_READ = 1ull << 1, RIGHT_FD_WRITE = 1ull << 6;

enum : uint8_t { FT_UNKNOWN = 0, FT_CHAR = 2, FT_DIR = 3, FT_FILE = 4, FT_SYMLINK = 7 };

uint32_t map_errno(int e) {
  switch (e) {
    case ENOENT: return W_ENOENT;
    case EACCES: return W_EACCES;
    case EEXIST: return W_EEXIST;
    case EISDIR: return W_EISDIR;
    case ENOTDIR: return W_ENOTDIR;
    case ENOTEMPTY: return W_ENOTEMPTY;
    case ELOOP: return W_ELOOP;
    case ENAMETOOLONG: return W_ENAMETOOLONG;
    case EINVAL: return W_EINVAL;
    case ENOSPC: return W_ENOSPC;
    case EPERM: return W_EPERM;
    case EBADF: return W_EBADF;
    case ESPIPE: return W_ESPIPE;
    default: return W_EIO;
  }
}

uint8_t filetype_of(mode_t m) {
  if (S_ISREG(m)) return FT_FILE;
  if (S_ISDIR(m)) return FT_DIR;
  if (S_ISCHR(m)) return FT_CHAR;
  if (S_ISLNK(m)) return FT_SYMLINK;
  return FT_UNKNOWN;
}

struct Fd {
  enum Kind { In, Out, Err, Dir, File } kind;
  std::string host;   // directory: host path (realpath)
  std::string guest;  // preopen name
  bool read_only = false;
  bool preopen = false;
  int os = -1;        // file: host descriptor
  bool can_read = false, can_write = false;
};

struct Wasi {
  const WasiConfig& cfg;
  WasiResult& res;
  size_t in_pos = 0;
  std::map<uint32_t, Fd> fds;
  std::mt19937_64 rng{std::random_device{}()};

  Wasi(const WasiConfig& c, WasiResult& r) : cfg(c), res(r) {
    fds[0] = Fd{Fd::In};
    fds[1] = Fd{Fd::Out};
    fds[2] = Fd{Fd::Err};
    uint32_t next = 3;
    for (auto& [host, guest, ro] : cfg.preopens) {
      char buf[PATH_MAX];
      if (!realpath(host.c_str(), buf)) throw LoadError("preopened directory does not exist: " + host);
      Fd d{Fd::Dir};
      d.host = buf;
      d.guest = guest;
      d.read_only = ro;
      d.preopen = true;
      fds[next++] = d;
    }
  }
  ~Wasi() {
    for (auto& [n, f] : fds)
      if (f.os >= 0) ::close(f.os);
  }

  Fd* fd(uint32_t n) {
    auto it = fds.find(n);
    return it == fds.end() ? nullptr : &it->second;
  }
  uint32_t alloc(Fd f) {
    uint32_t n = 3;
    while (fds.count(n)) ++n;
    fds[n] = std::move(f);
    return n;
  }

  // Host path for `rel` under directory `d`; refuses escapes.  With `parent_only`
  // only the parent has to exist (the last component may be created).
  uint32_t resolve(const Fd& d, const std::string& rel, std::string& out) {
    if (rel.empty() || rel.size() > 4096 || rel[0] == '/' || rel.find('\0') != std::string::npos) return W_ENOTCAPABLE;
    std::vector<std::string> parts;
    size_t i = 0;
    while (i <= rel.size()) {
      const size_t j = std::min(rel.find('/', i), rel.size());
      const std::string c = rel.substr(i, j - i);
      if (c == "..") return W_ENOTCAPABLE;
      if (!c.empty() && c != ".") parts.push_back(c);
      i = j + 1;
    }
    std::string parent = d.host;
    for (size_t k = 0; k + 1 < parts.size(); ++k) parent += "/" + parts[k];
    if (parts.empty()) {
      out = d.host;
      return W_OK_;
    }
    char buf[PATH_MAX];
    if (!realpath(parent.c_str(), buf)) return map_errno(errno);
    const std::string real_parent = buf;
    if (real_parent != d.host && real_parent.compare(0, d.host.size() + 1, d.host + "/") != 0) return W_ENOTCAPABLE;
    out = real_parent + "/" + parts.back();
    return W_OK_;
  }

  std::string guest_str(Instance& in, uint64_t ptr, uint64_t len) {
    return std::string(reinterpret_cast<const char*>(in.mem(ptr, len)), len);
  }
};

template <class T>
void put(Instance& in, uint64_t addr, T v) {
  std::memcpy(in.mem(addr, sizeof(T)), &v, sizeof(T));
}
template <class T>
T get(Instance& in, uint64_t addr) {
  T v;
  std::memcpy(&v, in.mem(addr, sizeof(T)), sizeof(T));
  return v;
}

void write_filestat(Instance& in, uint64_t p, const struct stat& s) {
  uint8_t* b = in.mem(p, 64);
  std::memset(b, 0, 64);
  const uint64_t dev = s.st_dev, ino = s.st_ino, nlink = s.st_nlink, size = s.st_size;
  const uint64_t at = (uint64_t)s.st_atim.tv_sec * 1000000000ull + s.st_atim.tv_nsec;
  const uint64_t mt = (uint64_t)s.st_mtim.tv_sec * 1000000000ull + s.st_mtim.tv_nsec;
  const uint64_t ct = (uint64_t)s.st_ctim.tv_sec * 1000000000ull + s.st_ctim.tv_nsec;
  std::memcpy(b + 0, &dev, 8);
  std::memcpy(b + 8, &ino, 8);
  b[16] = filetype_of(s.st_mode);
  std::memcpy(b + 24, &nlink, 8);
  std::memcpy(b + 32, &size, 8);
  std::memcpy(b + 40, &at, 8);
  std::memcpy(b + 48, &mt, 8);
  std::memcpy(b + 56, &ct, 8);
}

using A = const uint64_t*;
using R = uint64_t*;
#define ARG32(i) ((uint32_t)a[i])
#define RET(v) (r[0] = (uint32_t)(v))

struct Sig {
  const char* params;  // 'i' i32, 'I' i64
  bool ret;            // one i32 result
};

const std::map<std::string, Sig>& wasi_sigs() {
  static const std::map<std::string, Sig> m = {
      {"args_get", {"ii", true}},
      {"args_sizes_get", {"ii", true}},
      {"environ_get", {"ii", true}},
      {"environ_sizes_get", {"ii", true}},
      {"clock_res_get", {"ii", true}},
      {"clock_time_get", {"iIi", true}},
      {"fd_close", {"i", true}},
      {"fd_fdstat_get", {"ii", true}},
      {"fd_fdstat_set_flags", {"ii", true}},
      {"fd_filestat_get", {"ii", true}},
      {"fd_prestat_get", {"ii", true}},
      {"fd_prestat_dir_name", {"iii", true}},
      {"fd_read", {"iiii", true}},
      {"fd_readdir", {"iiiIi", true}},
      {"fd_seek", {"iIii", true}},
      {"fd_tell", {"ii", true}},
      {"fd_write", {"iiii", true}},
      {"fd_sync", {"i", true}},
      {"fd_datasync", {"i", true}},
      {"path_create_directory", {"iii", true}},
      {"path_filestat_get", {"iiiii", true}},
      {"path_open", {"iiiiiIIii", true}},
      {"path_remove_directory", {"iii", true}},
      {"path_unlink_file", {"iii", true}},
      {"proc_exit", {"i", false}},
      {"random_get", {"ii", true}},
      {"sched_yield", {"", true}},
  };
  return m;
}

bool sig_matches(const Sig& s, const FuncType& t) {
  const size_t n = std::strlen(s.params);
  if (t.params.size() != n) return false;
  for (size_t i = 0; i < n; ++i)
    if (t.params[i] != (s.params[i] == 'I' ? I64 : I32)) return false;
  return s.ret ? (t.results.size() == 1 && t.results[0] == I32) : t.results.empty();
}

HostFn bind(Wasi& w, const std::string& name) {
  if (name == "args_sizes_get" || name == "environ_sizes_get") {
    const bool env = name[0] == 'e';
    return [&w, env](Instance& in, A a, R r) {
      uint32_t count = 0, bytes = 0;
      if (env) {
        for (auto& [k, v] : w.cfg.env) ++count, bytes += (uint32_t)(k.size() + v.size() + 2);
      } else {
        for (auto& s : w.cfg.args) ++count, bytes += (uint32_t)(s.size() + 1);
      }
      put<uint32_t>(in, ARG32(0), count);
      put<uint32_t>(in, ARG32(1), bytes);
      RET(W_OK_);
    };
  }
  if (name == "args_get" || name == "environ_get") {
    const bool env = name[0] == 'e';
    return [&w, env](Instance& in, A a, R r) {
      uint32_t ptrs = ARG32(0), buf = ARG32(1);
      auto emit = [&](const std::string& s) {
        put<uint32_t>(in, ptrs, buf);
        ptrs += 4;
        std::memcpy(in.mem(buf, s.size() + 1), s.c_str(), s.size() + 1);
        buf += (uint32_t)s.size() + 1;
      };
      if (env) {
        for (auto& [k, v] : w.cfg.env) emit(k + "=" + v);
      } else {
        for (auto& s : w.cfg.args) emit(s);
      }
      RET(W_OK_);
    };
  }
  if (name == "clock_res_get") {
    return [](Instance& in, A a, R r) {
      put<uint64_t>(in, ARG32(1), 1);
      RET(W_OK_);
    };
  }
  if (name == "clock_time_get") {
    return [](Instance& in, A a, R r) {
      const uint32_t id = ARG32(0);
      timespec ts;
      clock_gettime(id == 0 ? CLOCK_REALTIME : CLOCK_MONOTONIC, &ts);
      put<uint64_t>(in, ARG32(2), (uint64_t)ts.tv_sec * 1000000000ull + (uint64_t)ts.tv_nsec);
      RET(W_OK_);
    };
  }
  if (name == "random_get") {
    return [&w](Instance& in, A a, R r) {
      uint8_t* p = in.mem(ARG32(0), ARG32(1));
      for (uint32_t i = 0; i < ARG32(1); ++i) p[i] = (uint8_t)w.rng();
      RET(W_OK_);
    };
  }
  if (name == "proc_exit") {
    return [](Instance&, A a, R) { throw ProcExit{(int32_t)ARG32(0)}; };
  }
  if (name == "sched_yield") {
    return [](Instance&, A, R r) { RET(W_OK_); };
  }
  if (name == "fd_read" || name == "fd_write") {
    const bool wr = name == "fd_write";
    return [&w, wr](Instance& in, A a, R r) {
      Fd* f = w.fd(ARG32(0));
      if (!f) return (void)RET(W_EBADF);
      const uint32_t iovs = ARG32(1), n = ARG32(2);
      uint64_t total = 0;
      for (uint32_t k = 0; k < n; ++k) {
        const uint32_t buf = get<uint32_t>(in, iovs + 8ull * k), len = get<uint32_t>(in, iovs + 8ull * k + 4);
        uint8_t* p = in.mem(buf, len);
        if (wr) {
          std::string* sink = f->kind == Fd::Out ? &w.res.out : f->kind == Fd::Err ? &w.res.err : nullptr;
          if (sink) {
            const size_t cap = f->kind == Fd::Out ? w.cfg.stdout_cap : w.cfg.stderr_cap;
            const size_t room = cap > sink->size() ? cap - sink->size() : 0;
            if (room == 0 && len) {
              if (total) break;
              return (void)RET(W_ENOSPC);
            }
            const size_t m = std::min<size_t>(room, len);
            sink->append(reinterpret_cast<const char*>(p), m);
            total += m;
            if (m < len) break;
          } else if (f->kind == Fd::File && f->can_write) {
            const ssize_t m = ::write(f->os, p, len);
            if (m < 0) return (void)RET(map_errno(errno));
            total += (uint64_t)m;
            if ((uint32_t)m < len) break;
          } else {
            return (void)RET(W_EBADF);
          }
        } else {
          if (f->kind == Fd::In) {
            const size_t m = std::min<size_t>(len, w.cfg.stdin_data.size() - w.in_pos);
            std::memcpy(p, w.cfg.stdin_data.data() + w.in_pos, m);
            w.in_pos += m;
            total += m;
            if (m < len) break;
          } else if (f->kind == Fd::File && f->can_read) {
            const ssize_t m = ::read(f->os, p, len);
            if (m < 0) return (void)RET(map_errno(errno));
            total += (uint64_t)m;
            if ((uint32_t)m < len) break;
          } else {
            return (void)RET(f->kind == Fd::Dir ? W_EISDIR : W_EBADF);
          }
        }
      }
      put<uint32_t>(in, ARG32(3), (uint32_t)total);
      RET(W_OK_);
    };
  }
  if (name == "fd_seek" || name == "fd_tell") {
    const bool tell = name == "fd_tell";
    return [&w, tell](Instance& in, A a, R r) {
      Fd* f = w.fd(ARG32(0));
      if (!f) return (void)RET(W_EBADF);
      if (f->kind != Fd::File) return (void)RET(f->kind == Fd::Dir ? W_EBADF : W_ESPIPE);
      off_t pos;
      if (tell) {
        pos = ::lseek(f->os, 0, SEEK_CUR);
      } else {
        const uint32_t wh = ARG32(2) & 0xff;
        if (wh > 2) return (void)RET(W_EINVAL);
        pos = ::lseek(f->os, (off_t)(int64_t)a[1], wh == 0 ? SEEK_SET : wh == 1 ? SEEK_CUR : SEEK_END);
      }
      if (pos < 0) return (void)RET(map_errno(errno));
      put<uint64_t>(in, tell ? ARG32(1) : ARG32(3), (uint64_t)pos);
      RET(W_OK_);
    };
  }
  if (name == "fd_close") {
    return [&w](Instance&, A a, R r) {
      auto it = w.fds.find(ARG32(0));
      if (it == w.fds.end()) return (void)RET(W_EBADF);
      if (it->second.os >= 0) ::close(it->second.os);
      w.fds.erase(it);
      RET(W_OK_);
    };
  }
  if (name == "fd_sync" || name == "fd_datasync" || name == "fd_fdstat_set_flags") {
    return [&w](Instance&, A a, R r) { RET(w.fd(ARG32(0)) ? W_OK_ : W_EBADF); };
  }
  if (name == "fd_fdstat_get") {
    return [&w](Instance& in, A a, R r) {
      Fd* f = w.fd(ARG32(0));
      if (!f) return (void)RET(W_EBADF);
      uint8_t* b = in.mem(ARG32(1), 24);
      std::memset(b, 0, 24);
      uint64_t base = 0, inh = 0;
      switch (f->kind) {
        case Fd::In: b[0] = FT_CHAR; base = RIGHT_FD_READ | (1ull << 27); break;
        case Fd::Out: case Fd::Err: b[0] = FT_CHAR; base = RIGHT_FD_WRITE | (1ull << 27); break;
        case Fd::Dir:
          b[0] = FT_DIR;
          base = inh = f->read_only ? RIGHTS_ALL & ~RIGHTS_MUTATE : RIGHTS_ALL;
          break;
        case Fd::File:
          b[0] = FT_FILE;
          base = RIGHTS_ALL & ~RIGHTS_MUTATE & ~RIGHT_FD_READ;
          if (f->can_read) base |= RIGHT_FD_READ;
          if (f->can_write) base |= RIGHT_FD_WRITE | (1ull << 22) | (1ull << 4) | (1ull << 0);
          break;
      }
      std::memcpy(b + 8, &base, 8);
      std::memcpy(b + 16, &inh, 8);
      RET(W_OK_);
    };
  }
  if (name == "fd_filestat_get") {
    return [&w](Instance& in, A a, R r) {
      Fd* f = w.fd(ARG32(0));
      if (!f) return (void)RET(W_EBADF);
      struct stat s {};
      if (f->kind == Fd::File) {
        if (fstat(f->os, &s) != 0) return (void)RET(map_errno(errno));
      } else if (f->kind == Fd::Dir) {
        if (stat(f->host.c_str(), &s) != 0) return (void)RET(map_errno(errno));
      } else {
        s.st_mode = S_IFCHR;
      }
      write_filestat(in, ARG32(1), s);
      RET(W_OK_);
    };
  }
  if (name == "fd_prestat_get") {
    return [&w](Instance& in, A a, R r) {
      Fd* f = w.fd(ARG32(0));
      if (!f || !f->preopen) return (void)RET(W_EBADF);
      put<uint32_t>(in, ARG32(1), 0);  // tag: directory
      put<uint32_t>(in, ARG32(1) + 4ull, (uint32_t)f->guest.size());
      RET(W_OK_);
    };
  }
  if (name == "fd_prestat_dir_name") {
    return [&w](Instance& in, A a, R r) {
      Fd* f = w.fd(ARG32(0));
      if (!f || !f->preopen) return (void)RET(W_EBADF);
      if (ARG32(2) < f->guest.size()) return (void)RET(W_EINVAL);
      std::memcpy(in.mem(ARG32(1), f->guest.size()), f->guest.data(), f->guest.size());
      RET(W_OK_);
    };
  }
  if (name == "fd_readdir") {
    return [&w](Instance& in, A a, R r) {
      Fd* f = w.fd(ARG32(0));
      if (!f) return (void)RET(W_EBADF);
      if (f->kind != Fd::Dir) return (void)RET(W_ENOTDIR);
      DIR* d = opendir(f->host.c_str());
      if (!d) return (void)RET(map_errno(errno));
      std::vector<std::pair<std::string, std::pair<uint64_t, uint8_t>>> ents;
      while (dirent* e = readdir(d)) {
        uint8_t t = e->d_type == DT_DIR ? FT_DIR : e->d_type == DT_REG ? FT_FILE : e->d_type == DT_LNK ? FT_SYMLINK
                                                                                                    : FT_UNKNOWN;
        ents.push_back({e->d_name, {(uint64_t)e->d_ino, t}});
      }
      closedir(d);
      std::sort(ents.begin(), ents.end());
      const uint32_t buf = ARG32(1), len = ARG32(2);
      uint8_t* out = in.mem(buf, len);
      uint64_t used = 0;
      for (uint64_t k = a[3]; k < ents.size() && used < len; ++k) {
        uint8_t hdr[24] = {};
        const uint64_t next = k + 1;
        const uint32_t nl = (uint32_t)ents[k].first.size();
        std::memcpy(hdr, &next, 8);
        std::memcpy(hdr + 8, &ents[k].second.first, 8);
        std::memcpy(hdr + 16, &nl, 4);
        hdr[20] = ents[k].second.second;
        std::string rec(reinterpret_cast<const char*>(hdr), 24);
        rec += ents[k].first;
        const uint64_t m = std::min<uint64_t>(rec.size(), len - used);  // a full buffer signals "more"
        std::memcpy(out + used, rec.data(), m);
        used += m;
      }
      put<uint32_t>(in, ARG32(4), (uint32_t)used);
      RET(W_OK_);
    };
  }
  if (name == "path_open") {
    return [&w](Instance& in, A a, R r) {
      Fd* d = w.fd(ARG32(0));
      if (!d) return (void)RET(W_EBADF);
      if (d->kind != Fd::Dir) return (void)RET(W_ENOTDIR);
      const std::string rel = w.guest_str(in, ARG32(2), ARG32(3));
      const uint32_t oflags = ARG32(4), fdflags = ARG32(7);
      const uint64_t rights = a[5];
      std::string path;
      if (uint32_t e = w.resolve(*d, rel, path)) return (void)RET(e);
      const bool creat = oflags & 1, want_dir = oflags & 2, excl = oflags & 4, trunc = oflags & 8;
      const bool append = fdflags & 1;
      const bool want_write = (rights & RIGHT_FD_WRITE) || append || trunc || creat;
      const bool want_read = (rights & RIGHT_FD_READ) || !want_write;
      if (d->read_only && (creat || trunc || excl || append || (rights & RIGHT_FD_WRITE)))
        return (void)RET(W_ENOTCAPABLE);
      struct stat s {};
      const bool exists = lstat(path.c_str(), &s) == 0;
      if (exists && S_ISLNK(s.st_mode)) return (void)RET(W_ELOOP);  // symlinks are not followed
      if (want_dir || (exists && S_ISDIR(s.st_mode))) {
        if (!exists) return (void)RET(W_ENOENT);
        if (!S_ISDIR(s.st_mode)) return (void)RET(W_ENOTDIR);
        if (want_write && !want_dir) return (void)RET(W_EISDIR);
        Fd nd{Fd::Dir};
        nd.host = path;
        nd.read_only = d->read_only;
        put<uint32_t>(in, ARG32(8), w.alloc(nd));
        return (void)RET(W_OK_);
      }
      int flags = O_CLOEXEC | O_NOFOLLOW;
      flags |= want_write ? (want_read ? O_RDWR : O_WRONLY) : O_RDONLY;
      if (creat) flags |= O_CREAT;
      if (excl) flags |= O_EXCL;
      if (trunc) flags |= O_TRUNC;
      if (append) flags |= O_APPEND;
      const int os = ::open(path.c_str(), flags, 0644);
      if (os < 0) return (void)RET(map_errno(errno));
      Fd nf{Fd::File};
      nf.os = os;
      nf.can_read = want_read;
      nf.can_write = want_write;
      nf.read_only = d->read_only;
      put<uint32_t>(in, ARG32(8), w.alloc(nf));
      RET(W_OK_);
    };
  }
  if (name == "path_filestat_get") {
    return [&w](Instance& in, A a, R r) {
      Fd* d = w.fd(ARG32(0));
      if (!d) return (void)RET(W_EBADF);
      if (d->kind != Fd::Dir) return (void)RET(W_ENOTDIR);
      std::string path;
      if (uint32_t e = w.resolve(*d, w.guest_str(in, ARG32(2), ARG32(3)), path)) return (void)RET(e);
      struct stat s {};
      if (lstat(path.c_str(), &s) != 0) return (void)RET(map_errno(errno));
      write_filestat(in, ARG32(4), s);
      RET(W_OK_);
    };
  }
  if (name == "path_create_directory" || name == "path_remove_directory" || name == "path_unlink_file") {
    const char op = name[5] == 'c' ? 'c' : name[5] == 'r' ? 'r' : 'u';
    return [&w, op](Instance& in, A a, R r) {
      Fd* d = w.fd(ARG32(0));
      if (!d) return (void)RET(W_EBADF);
      if (d->kind != Fd::Dir) return (void)RET(W_ENOTDIR);
      if (d->read_only) return (void)RET(W_ENOTCAPABLE);
      std::string path;
      if (uint32_t e = w.resolve(*d, w.guest_str(in, ARG32(1), ARG32(2)), path)) return (void)RET(e);
      if (path == d->host) return (void)RET(W_EPERM);
      const int rc = op == 'c' ? mkdir(path.c_str(), 0755) : op == 'r' ? rmdir(path.c_str()) : unlink(path.c_str());
      RET(rc == 0 ? W_OK_ : map_errno(errno));
    };
  }
  return {};
}

}  // namespace

WasiResult run_wasi(const std::string& module_bytes, const WasiConfig& cfg, RunLimits lim) {
  WasiResult res;
  Wasi w(cfg, res);
  Module m = Module::parse(module_bytes);
  auto host = [&w](const std::string& mod, const std::string& name, const FuncType& t) -> HostFn {
    if (mod != "wasi_snapshot_preview1" && mod != "wasi_unstable") return {};
    auto it = wasi_sigs().find(name);
    if (it == wasi_sigs().end()) {
      // other preview1 calls (sockets, poll, links, ...): callable, answer ENOSYS
      if (t.results.size() == 1 && t.results[0] == I32) return [](Instance&, A, R r) { RET(W_ENOSYS); };
      return {};
    }
    if (!sig_matches(it->second, t)) throw LoadError("WASI import " + name + " has the wrong signature");
    return bind(w, name);
  };
  try {
    Instance inst(std::move(m), host, lim);
    inst.invoke("_start", {});
  } catch (const ProcExit& e) {
    res.exit_code = e.code;
  }
  return res;
}

#undef ARG32
#undef RET

}  // namespace wasm
}  // namespace kapsl

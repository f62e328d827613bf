// kapsl_sdk.kapsl_sdk: the Python client SDK (C++).
//
// Same classes, signatures, defaults and exception mapping as the reference
// PyO3 module (crates/kapsl-pyo3/src/lib.rs:22-719, shm_client.rs,
// hybrid_client.rs):
//   KapslClient(endpoint=None, *, protocol=None, host=None, port=None,
//               socket_path=None, pipe_name=None, max_pool_size=8, api_token=None)
//     .protocol() .endpoint() .infer() .infer_tensor() .infer_stream()
//   KapslShmClient(shm_name).infer(shape, dtype, data)
//   KapslHybridClient(shm_name, socket_path).infer(shape, dtype, data)
// Errors: socket I/O -> ConnectionError; bad endpoint or dtype -> ValueError;
// server error frames and codec errors -> RuntimeError; SHM wait -> TimeoutError.
// Unary calls use pooled connections and retry once on a fresh connection
// after an I/O error; streams use a dedicated connection.
#include <arpa/inet.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <time.h>
#include <unistd.h>

#include <chrono>
#include <cstring>
#include <deque>
#include <map>
#include <mutex>
#include <optional>
#include <random>
#include <thread>

#include "netio.h"
#include "shm.h"
#include "wire.h"

namespace py = pybind11;
using namespace kapsl;

namespace {

constexpr const char* kDefaultSocket = "/tmp/kapsl.sock";
constexpr const char* kDefaultHost = "127.0.0.1";
constexpr int kDefaultPort = 9096;

struct IoError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

[[noreturn]] void raise_py(PyObject* type, const std::string& msg) {
  PyErr_SetString(type, msg.c_str());
  throw py::error_already_set();
}

std::optional<std::string> norm(const std::optional<std::string>& v) {
  if (!v) return std::nullopt;
  std::string s = *v;
  size_t a = s.find_first_not_of(" \t\r\n"), b = s.find_last_not_of(" \t\r\n");
  if (a == std::string::npos) return std::nullopt;
  return s.substr(a, b - a + 1);
}

bool starts_with(const std::string& s, const std::string& p) { return s.compare(0, p.size(), p) == 0; }

struct Target {
  bool tcp = false;
  std::string addr;  // socket path or host:port
};

Target from_endpoint(const std::string& ep) {
  if (ep.empty()) raise_py(PyExc_ValueError, "Endpoint cannot be empty");
  if (starts_with(ep, "tcp://")) {
    std::string a = ep.substr(6);
    if (a.empty()) raise_py(PyExc_ValueError, "tcp:// endpoint must include host:port");
    return {true, a};
  }
  if (starts_with(ep, "unix://")) {
    std::string p = ep.substr(7);
    if (p.empty()) raise_py(PyExc_ValueError, "unix:// endpoint must include a socket path");
    return {false, p};
  }
  return {false, ep};
}

Target resolve(std::optional<std::string> endpoint, std::optional<std::string> protocol,
               std::optional<std::string> host, std::optional<int> port, std::optional<std::string> socket_path,
               std::optional<std::string> pipe_name) {
  endpoint = norm(endpoint);
  protocol = norm(protocol);
  host = norm(host);
  socket_path = norm(socket_path);
  pipe_name = norm(pipe_name);
  if (protocol) {
    std::string p = *protocol;
    for (auto& c : p) c = (char)std::tolower((unsigned char)c);
    if (p == "tcp") {
      if (socket_path || pipe_name)
        raise_py(PyExc_ValueError, "protocol='tcp' cannot be combined with socket_path or pipe_name");
      if (endpoint) {
        if (host || port) raise_py(PyExc_ValueError, "When endpoint is provided, do not also pass host/port");
        if (starts_with(*endpoint, "tcp://")) {
          std::string a = endpoint->substr(6);
          if (a.empty()) raise_py(PyExc_ValueError, "tcp:// endpoint must include host:port");
          return {true, a};
        }
        if (endpoint->find("://") != std::string::npos)
          raise_py(PyExc_ValueError, "protocol='tcp' expects endpoint as host:port or tcp://host:port");
        return {true, *endpoint};
      }
      return {true, host.value_or(kDefaultHost) + ":" + std::to_string(port.value_or(kDefaultPort))};
    }
    if (p == "socket" || p == "unix" || p == "local") {
      if (host || port || pipe_name)
        raise_py(PyExc_ValueError, "protocol='socket' cannot be combined with host/port/pipe_name");
      if (socket_path) return from_endpoint(*socket_path);
      if (endpoint) return from_endpoint(*endpoint);
      return {false, kDefaultSocket};
    }
    if (p == "pipe" || p == "named_pipe" || p == "named-pipe") {
      if (host || port || socket_path)
        raise_py(PyExc_ValueError, "protocol='pipe' cannot be combined with host/port/socket_path");
      raise_py(PyExc_ValueError, "protocol='pipe' is only supported on Windows");
    }
    raise_py(PyExc_ValueError, "Unsupported protocol '" + p + "'. Use one of: socket, tcp, pipe");
  }
  if (endpoint) return from_endpoint(*endpoint);
  if (host || port) return {true, host.value_or(kDefaultHost) + ":" + std::to_string(port.value_or(kDefaultPort))};
  if (socket_path) return from_endpoint(*socket_path);
  if (pipe_name) raise_py(PyExc_ValueError, "pipe_name is only supported on Windows");
  return {false, kDefaultSocket};
}

int connect_target(const Target& t) {
  if (!t.tcp) {
    int fd = socket(AF_UNIX, SOCK_STREAM, 0);
    if (fd < 0) throw IoError("socket() failed");
    sockaddr_un a{};
    a.sun_family = AF_UNIX;
    std::strncpy(a.sun_path, t.addr.c_str(), sizeof(a.sun_path) - 1);
    if (connect(fd, reinterpret_cast<sockaddr*>(&a), sizeof(a)) != 0) {
      std::string e = std::string(strerror(errno)) + " (" + t.addr + ")";
      close(fd);
      throw IoError(e);
    }
    return fd;
  }
  const size_t colon = t.addr.rfind(':');
  if (colon == std::string::npos) throw IoError("invalid tcp address " + t.addr);
  std::string host = t.addr.substr(0, colon), port = t.addr.substr(colon + 1);
  addrinfo hints{}, *res = nullptr;
  hints.ai_family = AF_UNSPEC;
  hints.ai_socktype = SOCK_STREAM;
  if (getaddrinfo(host.c_str(), port.c_str(), &hints, &res) != 0 || !res) throw IoError("cannot resolve " + t.addr);
  int fd = -1;
  for (addrinfo* p = res; p; p = p->ai_next) {
    fd = socket(p->ai_family, p->ai_socktype, p->ai_protocol);
    if (fd < 0) continue;
    if (connect(fd, p->ai_addr, p->ai_addrlen) == 0) break;
    close(fd);
    fd = -1;
  }
  freeaddrinfo(res);
  if (fd < 0) throw IoError(std::string("connection refused (") + t.addr + ")");
  int one = 1;
  setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
  return fd;
}

std::string canon_dtype(const std::string& dt) {
  std::string c;
  int sz;
  if (!wire::dtype_parse(dt, &c, &sz)) raise_py(PyExc_ValueError, "Invalid input: Unsupported dtype: " + dt);
  return c;
}

std::vector<wire::NamedTensor> parse_extra(const std::optional<py::dict>& extra) {
  std::vector<wire::NamedTensor> out;
  if (!extra) return out;
  for (auto kv : *extra) {
    py::tuple t = kv.second.cast<py::tuple>();
    wire::NamedTensor nt;
    nt.name = kv.first.cast<std::string>();
    for (auto d : t[0]) nt.tensor.shape.push_back(d.cast<int64_t>());
    nt.tensor.dtype = canon_dtype(t[1].cast<std::string>());
    nt.tensor.data = t[2].cast<std::string>();
    out.push_back(std::move(nt));
  }
  return out;
}

struct Frame {
  uint32_t status;
  std::string payload;
};

Frame read_frame(int fd) {
  uint8_t h[8];
  if (!net::read_exact(fd, h, 8)) throw IoError("connection closed by server");
  Frame f;
  uint32_t size;
  std::memcpy(&f.status, h, 4);
  std::memcpy(&size, h + 4, 4);
  f.payload.resize(size);
  if (size && !net::read_exact(fd, f.payload.data(), size)) throw IoError("connection closed by server");
  return f;
}

class StreamIterator {
 public:
  explicit StreamIterator(int fd) : fd_(fd) {}
  ~StreamIterator() {
    if (fd_ >= 0) close(fd_);
  }
  py::bytes next() {
    if (fd_ < 0) throw py::stop_iteration();
    Frame f;
    {
      py::gil_scoped_release nogil;
      try {
        f = read_frame(fd_);
      } catch (const IoError& e) {
        py::gil_scoped_acquire g;
        finish();
        raise_py(PyExc_RuntimeError, e.what());
      }
    }
    if (f.status == wire::STATUS_STREAM_CHUNK && !f.payload.empty()) {
      try {
        return py::bytes(wire::decode_packet(f.payload).data);
      } catch (const std::exception& e) {
        raise_py(PyExc_RuntimeError, e.what());
      }
    }
    if (f.status == wire::STATUS_ERR && !f.payload.empty()) raise_py(PyExc_RuntimeError, f.payload);
    finish();
    throw py::stop_iteration();
  }

 private:
  void finish() {
    if (fd_ >= 0) close(fd_);
    fd_ = -1;
  }
  int fd_;
};

class KapslClient {
 public:
  KapslClient(std::optional<std::string> endpoint, std::optional<std::string> protocol,
              std::optional<std::string> host, std::optional<int> port, std::optional<std::string> socket_path,
              std::optional<std::string> pipe_name, size_t max_pool_size, std::optional<std::string> api_token)
      : target_(resolve(endpoint, protocol, host, port, socket_path, pipe_name)),
        max_pool_(max_pool_size),
        token_(api_token) {}
  ~KapslClient() {
    for (int fd : pool_) close(fd);
  }

  std::string protocol() const { return target_.tcp ? "tcp" : "socket"; }
  std::string endpoint() const { return (target_.tcp ? "tcp://" : "unix://") + target_.addr; }

  wire::Packet run(uint32_t model_id, std::vector<int64_t> shape, std::string dtype, std::string data,
                   std::optional<py::dict> extra, std::optional<std::string> session_id) {
    wire::Request req;
    req.input.shape = std::move(shape);
    req.input.dtype = canon_dtype(dtype);
    req.input.data = std::move(data);
    req.additional_inputs = parse_extra(extra);
    req.session_id = session_id;
    if (token_) {  // metadata is only sent when a token is set
      wire::Metadata m;
      m.auth_token = token_;
      req.metadata = m;
    }
    const std::string payload = wire::encode_request(req);
    py::gil_scoped_release nogil;
    int fd = -1;
    try {
      fd = checkout();
      Frame f = call(fd, model_id, wire::OP_INFER, payload);
      return finish_unary(fd, f);
    } catch (const IoError&) {
      if (fd >= 0) close(fd);
      fd = -1;
      try {
        fd = connect_target(target_);
        Frame f = call(fd, model_id, wire::OP_INFER, payload);
        return finish_unary(fd, f);
      } catch (const IoError& e2) {
        if (fd >= 0) close(fd);
        py::gil_scoped_acquire g;
        raise_py(PyExc_ConnectionError, e2.what());
      }
    }
  }

  py::bytes infer(uint32_t model_id, std::vector<int64_t> shape, std::string dtype, std::string data,
                  std::optional<py::dict> extra, std::optional<std::string> session_id) {
    wire::Packet p = run(model_id, std::move(shape), std::move(dtype), std::move(data), extra, session_id);
    return py::bytes(p.data);
  }

  py::tuple infer_tensor(uint32_t model_id, std::vector<int64_t> shape, std::string dtype, std::string data,
                         std::optional<py::dict> extra, std::optional<std::string> session_id) {
    wire::Packet p = run(model_id, std::move(shape), std::move(dtype), std::move(data), extra, session_id);
    return py::make_tuple(py::bytes(p.data), p.shape, p.dtype);
  }

  std::unique_ptr<StreamIterator> infer_stream(uint32_t model_id, std::vector<int64_t> shape, std::string dtype,
                                               std::string data, std::optional<py::dict> extra,
                                               std::optional<std::string> session_id) {
    wire::Request req;
    req.input.shape = std::move(shape);
    req.input.dtype = canon_dtype(dtype);
    req.input.data = std::move(data);
    req.additional_inputs = parse_extra(extra);
    req.session_id = session_id;
    if (token_) {
      wire::Metadata m;
      m.auth_token = token_;
      req.metadata = m;
    }
    const std::string payload = wire::encode_request(req);
    int fd;
    try {
      py::gil_scoped_release nogil;
      fd = connect_target(target_);
      std::string msg = wire::request_header(model_id, wire::OP_INFER_STREAM, (uint32_t)payload.size()) + payload;
      if (!net::write_all(fd, msg.data(), msg.size())) {
        close(fd);
        throw IoError("failed to send request");
      }
    } catch (const IoError& e) {
      raise_py(PyExc_ConnectionError, e.what());
    }
    return std::make_unique<StreamIterator>(fd);
  }

 private:
  int checkout() {
    {
      std::lock_guard<std::mutex> g(mu_);
      if (!pool_.empty()) {
        int fd = pool_.front();
        pool_.pop_front();
        return fd;
      }
    }
    return connect_target(target_);
  }
  void give_back(int fd) {
    if (max_pool_ > 0) {
      std::lock_guard<std::mutex> g(mu_);
      if (pool_.size() < max_pool_) {
        pool_.push_back(fd);
        return;
      }
    }
    close(fd);
  }
  static Frame call(int fd, uint32_t model_id, uint32_t op, const std::string& payload) {
    std::string msg = wire::request_header(model_id, op, (uint32_t)payload.size()) + payload;
    if (!net::write_all(fd, msg.data(), msg.size())) throw IoError("failed to send request");
    return read_frame(fd);
  }
  wire::Packet finish_unary(int fd, const Frame& f) {
    give_back(fd);
    if (f.status != wire::STATUS_OK) {
      py::gil_scoped_acquire g;
      raise_py(PyExc_RuntimeError, f.payload);
    }
    try {
      return wire::decode_packet(f.payload);
    } catch (const std::exception& e) {
      py::gil_scoped_acquire g;
      raise_py(PyExc_RuntimeError, e.what());
    }
  }

  Target target_;
  size_t max_pool_;
  std::optional<std::string> token_;
  std::mutex mu_;
  std::deque<int> pool_;
};

uint64_t now_ns() {
  return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
             std::chrono::system_clock::now().time_since_epoch())
      .count();
}

// Client-side leases use the lower half of the tensor pool (servers write
// results into the upper half) and are shared by every client of the region
// through lease words in header page 0, so two clients never write the same slot.
std::unique_ptr<shm::SharedLeases> client_allocator(shm::Region& r) {
  const auto& h = r.header();
  return std::make_unique<shm::SharedLeases>(r, h.tensor_pool_offset, h.max_tensor_size / 2);
}

// Request ids must not collide between client instances that share the
// response ring: start each client at a random 64-bit base.
uint64_t random_id_base() {
  std::random_device rd;
  uint64_t x = ((uint64_t)rd() << 32) ^ rd() ^ ((uint64_t)getpid() << 16) ^ now_ns();
  return (x | 1ull) & ~(1ull << 63);
}

class KapslShmClient {
 public:
  explicit KapslShmClient(const std::string& name) {
    try {
      region_ = std::make_unique<shm::Region>(shm::Region::open(name));
    } catch (const std::exception& e) {
      raise_py(PyExc_ConnectionError, e.what());
    }
    alloc_ = client_allocator(*region_);
  }

  py::bytes infer(std::vector<int64_t> shape, std::string dtype, std::string data) {
    wire::Packet p;
    p.shape = std::move(shape);
    p.dtype = canon_dtype(dtype);
    p.data = std::move(data);
    const uint64_t need = shm::tensor_bytes(p);
    auto off = alloc_->try_allocate(need);
    if (!off)
      raise_py(PyExc_RuntimeError, "SHM tensor pool exhausted (required=" + std::to_string(need) +
                                       " bytes, largest_slot=" + std::to_string(alloc_->largest_slot()) +
                                       " bytes, layout=" + alloc_->layout_summary() + ")");
    const uint64_t rid = next_id_++;
    std::string err;
    std::string result;
    bool timeout = false;
    {
      py::gil_scoped_release nogil;
      shm::write_tensor(*region_, *off, p);
      shm::ShmRequest q{};
      q.meta.request_id = rid;
      q.meta.model_id = 0;
      q.meta.priority = 0;
      q.meta.timestamp_ns = now_ns();
      q.tensor_offset = *off;
      q.tensor_size = need;
      shm::Ring<shm::ShmRequest> req(region_->base() + shm::REQ_RING_OFFSET, shm::RING_CAPACITY_ARG, false);
      if (!req.push(q)) {
        err = "Queue is full";
      } else {
        shm::Ring<shm::ShmResponse> resp(region_->base() + shm::RESP_RING_OFFSET, shm::RING_CAPACITY_ARG, false);
        const auto t0 = std::chrono::steady_clock::now();
        unsigned spins = 0;
        for (;;) {
          auto r = resp.pop();
          if (r) {
            if (r->meta.request_id != rid) {
              // another client's response: put it back (retry while the ring is full,
              // dropping it would leave its owner waiting until its timeout)
              while (!resp.push(*r) && std::chrono::steady_clock::now() - t0 < std::chrono::seconds(5))
                std::this_thread::yield();
            } else {
              if (r->meta.status != 0) {
                err = r->error_offset ? shm::read_error(*region_, r->error_offset) : "Unknown error";
                if (r->error_offset) shm::mark_result_read(*region_, r->error_offset);
              } else {
                wire::Packet out = shm::read_tensor(*region_, r->result_offset);
                result = std::move(out.data);
                shm::mark_result_read(*region_, r->result_offset);  // the server may reuse the slot now
              }
              break;
            }
          }
          if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(5)) {
            timeout = true;
            break;
          }
          if (++spins > 256) std::this_thread::sleep_for(std::chrono::microseconds(1));
        }
      }
      alloc_->release(*off);
    }
    if (timeout) raise_py(PyExc_TimeoutError, "Timed out waiting for SHM response");
    if (!err.empty()) raise_py(PyExc_RuntimeError, err);
    return py::bytes(result);
  }

 private:
  std::unique_ptr<shm::Region> region_;
  std::unique_ptr<shm::SharedLeases> alloc_;
  uint64_t next_id_ = random_id_base();
};

class KapslHybridClient {
 public:
  KapslHybridClient(const std::string& shm_name, const std::string& socket_path) : target_{false, socket_path} {
    try {
      region_ = std::make_unique<shm::Region>(shm::Region::open(shm_name));
    } catch (const std::exception& e) {
      raise_py(PyExc_ConnectionError, e.what());
    }
    alloc_ = client_allocator(*region_);
    try {
      fd_ = connect_target(target_);
    } catch (const IoError& e) {
      raise_py(PyExc_RuntimeError, e.what());
    }
  }
  ~KapslHybridClient() {
    if (fd_ >= 0) close(fd_);
  }

  py::bytes infer(std::vector<int64_t> shape, std::string dtype, std::string data) {
    wire::Packet p;
    p.shape = std::move(shape);
    p.dtype = canon_dtype(dtype);
    p.data = std::move(data);
    const uint64_t need = shm::tensor_bytes(p);
    auto off = alloc_->try_allocate(need);
    if (!off) raise_py(PyExc_RuntimeError, "SHM tensor pool exhausted (required=" + std::to_string(need) + " bytes)");
    wire::HybridRequest h;
    h.meta.request_id = next_id_++;
    h.meta.model_id = 0;
    h.meta.timestamp_ns = now_ns();
    h.shm_offset = *off;
    h.shm_size = need;
    Frame f;
    std::string io_err;
    {
      py::gil_scoped_release nogil;
      shm::write_tensor(*region_, *off, p);
      const std::string payload = wire::encode_hybrid_request(h);
      const std::string msg = wire::request_header(0, wire::OP_HYBRID_INFER, (uint32_t)payload.size()) + payload;
      try {
        if (!net::write_all(fd_, msg.data(), msg.size())) throw IoError("failed to send request");
        f = read_frame(fd_);
      } catch (const IoError& e) {
        io_err = e.what();
      }
      alloc_->release(*off);
    }
    if (!io_err.empty()) raise_py(PyExc_RuntimeError, io_err);
    if (f.status != wire::STATUS_OK) raise_py(PyExc_RuntimeError, f.payload);
    wire::HybridResponse r;
    try {
      r = wire::decode_hybrid_response(f.payload);
      std::string data = shm::read_tensor(*region_, r.shm_offset).data;
      shm::mark_result_read(*region_, r.shm_offset);  // the server may reuse the slot now
      return py::bytes(data);
    } catch (const std::exception& e) {
      raise_py(PyExc_RuntimeError, e.what());
    }
  }

 private:
  Target target_;
  std::unique_ptr<shm::Region> region_;
  std::unique_ptr<shm::SharedLeases> alloc_;
  int fd_ = -1;
  uint64_t next_id_ = random_id_base();
};

}  // namespace

PYBIND11_MODULE(kapsl_sdk, m) {
  m.doc() = "kapsl client SDK (C++): Unix socket / TCP / shared-memory / hybrid clients";
  py::class_<StreamIterator>(m, "StreamIterator")
      .def("__iter__", [](StreamIterator& s) -> StreamIterator& { return s; }, py::return_value_policy::reference_internal)
      .def("__next__", &StreamIterator::next);
  py::class_<KapslClient>(m, "KapslClient")
      .def(py::init<std::optional<std::string>, std::optional<std::string>, std::optional<std::string>,
                    std::optional<int>, std::optional<std::string>, std::optional<std::string>, size_t,
                    std::optional<std::string>>(),
           py::arg("endpoint") = py::none(), py::kw_only(), py::arg("protocol") = py::none(),
           py::arg("host") = py::none(), py::arg("port") = py::none(), py::arg("socket_path") = py::none(),
           py::arg("pipe_name") = py::none(), py::arg("max_pool_size") = 8, py::arg("api_token") = py::none())
      .def("protocol", &KapslClient::protocol)
      .def("endpoint", &KapslClient::endpoint)
      .def("infer", &KapslClient::infer, py::arg("model_id"), py::arg("shape"), py::arg("dtype"), py::arg("data"),
           py::arg("additional_inputs") = py::none(), py::arg("session_id") = py::none())
      .def("infer_tensor", &KapslClient::infer_tensor, py::arg("model_id"), py::arg("shape"), py::arg("dtype"),
           py::arg("data"), py::arg("additional_inputs") = py::none(), py::arg("session_id") = py::none())
      .def("infer_stream", &KapslClient::infer_stream, py::arg("model_id"), py::arg("shape"), py::arg("dtype"),
           py::arg("data"), py::arg("additional_inputs") = py::none(), py::arg("session_id") = py::none());
  py::class_<KapslShmClient>(m, "KapslShmClient")
      .def(py::init<std::string>(), py::arg("shm_name"))
      .def("infer", &KapslShmClient::infer, py::arg("shape"), py::arg("dtype"), py::arg("data"));
  py::class_<KapslHybridClient>(m, "KapslHybridClient")
      .def(py::init<std::string, std::string>(), py::arg("shm_name"), py::arg("socket_path"))
      .def("infer", &KapslHybridClient::infer, py::arg("shape"), py::arg("dtype"), py::arg("data"));
}

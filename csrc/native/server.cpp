#include "server.h"

#include <algorithm>
#include <arpa/inet.h>
#include <errno.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/socket.h>
#include <sys/stat.h>
#include <sys/un.h>
#include <unistd.h>

#include <chrono>
#include <cstring>

#include "netio.h"

namespace kapsl {

// --------------------------------------------------------- py conversions
py::tuple packet_to_py(const wire::Packet& p) {
  py::list shape;
  for (int64_t d : p.shape) shape.append(d);
  return py::make_tuple(shape, p.dtype, py::bytes(p.data));
}

wire::Packet packet_from_py(const py::handle& obj) {
  py::tuple t = py::reinterpret_borrow<py::object>(obj).cast<py::tuple>();
  if (t.size() != 3) throw std::runtime_error("handler must return (shape, dtype, data)");
  wire::Packet p;
  for (auto d : t[0]) p.shape.push_back(d.cast<int64_t>());
  std::string dt = t[1].cast<std::string>();
  int sz;
  if (!wire::dtype_parse(dt, &p.dtype, &sz)) throw std::runtime_error("Unsupported dtype: " + dt);
  p.data = t[2].cast<std::string>();
  return p;
}

py::dict request_to_py(const wire::Request& r) {
  py::dict d;
  d["input"] = packet_to_py(r.input);
  py::list extra;
  for (const auto& nt : r.additional_inputs) extra.append(py::make_tuple(nt.name, packet_to_py(nt.tensor)));
  d["additional_inputs"] = extra;
  d["session_id"] = r.session_id ? py::object(py::str(*r.session_id)) : py::object(py::none());
  if (r.metadata) {
    const auto& m = *r.metadata;
    py::dict md;
    auto put = [&](const char* k, auto v) {
      if (v.has_value())
        md[k] = *v;
      else
        md[k] = py::none();
    };
    put("request_id", m.request_id);
    put("timeout_ms", m.timeout_ms);
    if (m.priority)
      md["priority"] = (int)*m.priority;
    else
      md["priority"] = py::none();
    put("force_cpu", m.force_cpu);
    put("model_version", m.model_version);
    put("auth_token", m.auth_token);
    put("max_new_tokens", m.max_new_tokens);
    put("temperature", m.temperature);
    put("top_p", m.top_p);
    put("top_k", m.top_k);
    put("repetition_penalty", m.repetition_penalty);
    put("seed", m.seed);
    if (m.stop_token_ids) {
      py::list ids;
      for (uint32_t x : *m.stop_token_ids) ids.append(x);
      md["stop_token_ids"] = ids;
    } else {
      md["stop_token_ids"] = py::none();
    }
    d["metadata"] = md;
  } else {
    d["metadata"] = py::none();
  }
  return d;
}

static std::string py_error_message(py::error_already_set& e) {
  try {
    return py::str(e.value()).cast<std::string>();
  } catch (...) {
    return e.what();
  }
}

// ------------------------------------------------------------- WireServer
WireServer::WireServer(py::object handler, std::optional<std::string> auth_token)
    : handler_(std::move(handler)), token_(std::move(auth_token)) {}

WireServer::~WireServer() {
  py::gil_scoped_release nogil;
  stop();
}

void WireServer::listen_unix(const std::string& path) {
  // refuse a live socket, remove a stale one (crates/kapsl-ipc/src/server.rs:115-130)
  struct stat st;
  if (stat(path.c_str(), &st) == 0) {
    int probe = socket(AF_UNIX, SOCK_STREAM, 0);
    sockaddr_un a{};
    a.sun_family = AF_UNIX;
    std::strncpy(a.sun_path, path.c_str(), sizeof(a.sun_path) - 1);
    const bool live = connect(probe, reinterpret_cast<sockaddr*>(&a), sizeof(a)) == 0;
    close(probe);
    if (live) throw std::runtime_error("socket " + path + " is in use by a running server");
    unlink(path.c_str());
  }
  int fd = socket(AF_UNIX, SOCK_STREAM, 0);
  if (fd < 0) throw std::runtime_error("socket() failed");
  sockaddr_un a{};
  a.sun_family = AF_UNIX;
  if (path.size() >= sizeof(a.sun_path)) throw std::runtime_error("socket path too long");
  std::strncpy(a.sun_path, path.c_str(), sizeof(a.sun_path) - 1);
  if (bind(fd, reinterpret_cast<sockaddr*>(&a), sizeof(a)) != 0) {
    close(fd);
    throw std::runtime_error("bind(" + path + ") failed: " + strerror(errno));
  }
  chmod(path.c_str(), 0600);
  if (listen(fd, 512) != 0) {
    close(fd);
    throw std::runtime_error("listen failed");
  }
  unix_path_ = path;
  listen_fds_.push_back(fd);
}

int WireServer::listen_tcp(const std::string& host, int port) {
  int fd = socket(AF_INET, SOCK_STREAM, 0);
  if (fd < 0) throw std::runtime_error("socket() failed");
  int one = 1;
  setsockopt(fd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
  sockaddr_in a{};
  a.sin_family = AF_INET;
  a.sin_port = htons((uint16_t)port);
  if (inet_pton(AF_INET, host.c_str(), &a.sin_addr) != 1) {
    close(fd);
    throw std::runtime_error("invalid IPv4 host " + host);
  }
  if (bind(fd, reinterpret_cast<sockaddr*>(&a), sizeof(a)) != 0) {
    close(fd);
    throw std::runtime_error("bind tcp failed: " + std::string(strerror(errno)));
  }
  if (listen(fd, 512) != 0) {
    close(fd);
    throw std::runtime_error("listen failed");
  }
  socklen_t len = sizeof(a);
  getsockname(fd, reinterpret_cast<sockaddr*>(&a), &len);
  listen_fds_.push_back(fd);
  return ntohs(a.sin_port);
}

void WireServer::attach_shm(const std::string& shm_name) {
  hybrid_region_ = std::make_unique<shm::Region>(shm::Region::open(shm_name));
  const auto& h = hybrid_region_->header();
  // results go to the upper half of the tensor pool; clients write inputs into the lower half
  const uint64_t half = h.max_tensor_size / 2;
  hybrid_alloc_ = std::make_unique<shm::TieredAllocator>(h.tensor_pool_offset + half, h.max_tensor_size - half);
  hybrid_alloc_->set_guard(hybrid_region_->base());  // a result slot is reused only once its client read it
}

void WireServer::start() {
  if (running_.exchange(true)) return;
  for (int fd : listen_fds_) threads_.emplace_back([this, fd] { accept_loop(fd); });
}

void WireServer::stop() {
  if (!running_.exchange(false)) return;
  for (int fd : listen_fds_) shutdown(fd, SHUT_RDWR);
  for (auto& t : threads_)
    if (t.joinable()) t.join();
  threads_.clear();
  for (int fd : listen_fds_) close(fd);
  listen_fds_.clear();
  std::vector<Conn> conns;
  {
    std::lock_guard<std::mutex> g(conn_mu_);
    for (int fd : conn_fds_) shutdown(fd, SHUT_RDWR);
    conns.swap(conns_);
  }
  for (auto& c : conns)
    if (c.t.joinable()) c.t.join();
  if (!unix_path_.empty()) unlink(unix_path_.c_str());
}

void WireServer::accept_loop(int lfd) {
  while (running_.load()) {
    pollfd p{lfd, POLLIN, 0};
    int r = poll(&p, 1, 200);
    if (r <= 0) continue;
    int fd = accept(lfd, nullptr, nullptr);
    if (fd < 0) continue;
    int one = 1;
    setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
    std::lock_guard<std::mutex> g(conn_mu_);
    for (auto it = conns_.begin(); it != conns_.end();) {
      if (it->done->load()) {
        it->t.join();
        it = conns_.erase(it);
      } else {
        ++it;
      }
    }
    conn_fds_.push_back(fd);
    auto done = std::make_shared<std::atomic<bool>>(false);
    conns_.push_back(Conn{std::thread([this, fd, done] {
                            serve_connection(fd);
                            done->store(true);
                          }),
                          done});
  }
}

// Streams a token channel: every token queued since the last wake-up becomes an
// int32 [1, 1] chunk frame, written together in one call; then END (or ERR, END).
// A failed write (the client went away) cancels the channel, and the producer
// aborts the request.
bool WireServer::stream_channel(int fd, TokenChannel& ch) {
  std::vector<int32_t> toks;
  std::string cerr, out;
  for (;;) {
    const int st = ch.pop(toks, cerr, 200);
    if (st == TokenChannel::kTimeout) {
      if (!running_.load()) {
        ch.cancel();
        return false;
      }
      continue;
    }
    if (st == TokenChannel::kTokens) {
      out.clear();
      wire::Packet pk;
      pk.shape = {1, 1};
      pk.dtype = "int32";
      for (const int32_t t : toks) {
        pk.data.assign(reinterpret_cast<const char*>(&t), 4);
        const std::string pl = wire::encode_packet(pk);
        out += wire::response_header(wire::STATUS_STREAM_CHUNK, (uint32_t)pl.size());
        out += pl;
      }
      if (!net::write_all(fd, out.data(), out.size())) {
        ch.cancel();
        return false;
      }
      continue;
    }
    if (st == TokenChannel::kError) return send_frame(fd, wire::STATUS_ERR, cerr) && send_frame(fd, wire::STATUS_STREAM_END, "");
    return send_frame(fd, wire::STATUS_STREAM_END, "");
  }
}

bool WireServer::send_frame(int fd, uint32_t status, const std::string& payload) {
  std::string out = wire::response_header(status, (uint32_t)payload.size());
  out += payload;
  return net::write_all(fd, out.data(), out.size());
}

std::optional<std::string> WireServer::check_auth(const wire::Request& r) const {
  if (!token_) return std::nullopt;
  if (r.metadata && r.metadata->auth_token && *r.metadata->auth_token == *token_) return std::nullopt;
  return std::string("Unauthorized");
}

void WireServer::serve_connection(int fd) {
  constexpr uint32_t kMaxPayload = 1u << 31;
  while (running_.load()) {
    uint8_t hdr[12];
    if (!net::read_exact(fd, hdr, 12)) break;
    uint32_t model_id, op, size;
    std::memcpy(&model_id, hdr, 4);
    std::memcpy(&op, hdr + 4, 4);
    std::memcpy(&size, hdr + 8, 4);
    if (size > kMaxPayload) break;
    // grow the buffer with the bytes that actually arrive (1 MiB at a time), so a
    // header that declares a huge payload and sends nothing holds no memory for it
    std::string payload;
    bool complete = true;
    for (uint32_t got = 0; got < size;) {
      const uint32_t n = std::min<uint32_t>(size - got, 1u << 20);
      payload.resize((size_t)got + n);
      if (!net::read_exact(fd, payload.data() + got, n)) {
        complete = false;
        break;
      }
      got += n;
    }
    if (!complete) break;
    if (!handle_frame(fd, model_id, op, payload)) break;
    served_.fetch_add(1);
  }
  {
    std::lock_guard<std::mutex> g(conn_mu_);
    for (auto it = conn_fds_.begin(); it != conn_fds_.end(); ++it)
      if (*it == fd) {
        conn_fds_.erase(it);
        break;
      }
  }
  close(fd);
}

bool WireServer::handle_frame(int fd, uint32_t model_id, uint32_t op, const std::string& payload) {
  using namespace wire;
  if (op == OP_INFER) {
    Request req;
    try {
      req = decode_request(payload);
    } catch (const std::exception& e) {
      return send_frame(fd, STATUS_ERR, e.what());
    }
    if (auto err = check_auth(req)) return send_frame(fd, STATUS_ERR, *err);
    Packet out;
    std::string err;
    {
      py::gil_scoped_acquire gil;
      try {
        py::object res = handler_.attr("infer")(model_id, request_to_py(req), "throughput");
        out = packet_from_py(res);
      } catch (py::error_already_set& e) {
        err = py_error_message(e);
      } catch (const std::exception& e) {
        err = e.what();
      }
    }
    if (!err.empty()) return send_frame(fd, STATUS_ERR, err);
    return send_frame(fd, STATUS_OK, encode_packet(out));
  }
  if (op == OP_INFER_STREAM) {
    Request req;
    try {
      req = decode_request(payload);
    } catch (const std::exception& e) {
      return send_frame(fd, STATUS_ERR, e.what());
    }
    if (auto err = check_auth(req)) return send_frame(fd, STATUS_ERR, *err);
    py::object it;
    std::shared_ptr<TokenChannel> ch;
    std::string err;
    {
      py::gil_scoped_acquire gil;
      try {
        py::object res = handler_.attr("infer_stream")(model_id, request_to_py(req));
        if (py::isinstance<TokenChannel>(res))
          ch = res.cast<std::shared_ptr<TokenChannel>>();  // token ids streamed without the GIL
        else
          it = py::iter(res);
      } catch (py::error_already_set& e) {
        err = py_error_message(e);
      } catch (const std::exception& e) {
        err = e.what();
      }
    }
    if (!err.empty()) return send_frame(fd, STATUS_ERR, err);  // initial failure: ERR only
    if (ch) return stream_channel(fd, *ch);
    bool ok = true;
    for (;;) {
      Packet chunk;
      bool done = false;
      std::string mid_err;
      {
        py::gil_scoped_acquire gil;
        try {
          PyObject* nxt = PyIter_Next(it.ptr());
          if (nxt == nullptr) {
            if (PyErr_Occurred()) throw py::error_already_set();
            done = true;
          } else {
            py::object o = py::reinterpret_steal<py::object>(nxt);
            chunk = packet_from_py(o);
          }
        } catch (py::error_already_set& e) {
          mid_err = py_error_message(e);
        } catch (const std::exception& e) {
          mid_err = e.what();
        }
      }
      if (!mid_err.empty()) {
        ok = send_frame(fd, STATUS_ERR, mid_err) && send_frame(fd, STATUS_STREAM_END, "");
        break;
      }
      if (done) {
        ok = send_frame(fd, STATUS_STREAM_END, "");
        break;
      }
      if (!send_frame(fd, STATUS_STREAM_CHUNK, encode_packet(chunk))) {
        ok = false;  // client went away: close the generator so the request is cancelled
        break;
      }
    }
    {
      py::gil_scoped_acquire gil;
      try {
        if (py::hasattr(it, "close")) it.attr("close")();
      } catch (py::error_already_set&) {
      }
      it = py::object();
    }
    return ok;
  }
  if (op == OP_HYBRID_INFER) {
    HybridRequest hr;
    try {
      hr = decode_hybrid_request(payload);
    } catch (const std::exception& e) {
      return send_frame(fd, STATUS_ERR, e.what());
    }
    if (!hybrid_region_) return send_frame(fd, STATUS_ERR, "hybrid inference needs a shared memory region");
    const auto t0 = std::chrono::steady_clock::now();
    Packet in;
    try {
      in = shm::read_tensor(*hybrid_region_, hr.shm_offset);
    } catch (const std::exception& e) {
      return send_frame(fd, STATUS_ERR, e.what());
    }
    Request req;
    req.input = std::move(in);
    Packet out;
    std::string err;
    {
      py::gil_scoped_acquire gil;
      try {
        out = packet_from_py(handler_.attr("infer")(hr.meta.model_id, request_to_py(req), "latency"));
      } catch (py::error_already_set& e) {
        err = py_error_message(e);
      } catch (const std::exception& e) {
        err = e.what();
      }
    }
    if (!err.empty()) return send_frame(fd, STATUS_ERR, err);
    const uint64_t need = shm::tensor_bytes(out);
    auto slot = hybrid_alloc_->try_allocate(need + shm::kResultGuard, /*force=*/true);
    if (!slot) return send_frame(fd, STATUS_ERR, "SHM result pool exhausted (" + std::to_string(need) + " bytes)");
    *slot += shm::kResultGuard;  // the guard word sits in front of the tensor
    shm::write_tensor(*hybrid_region_, *slot, out);
    HybridResponse resp;
    resp.meta.request_id = hr.meta.request_id;
    resp.meta.status = 0;
    resp.meta.latency_ns =
        (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count();
    resp.shm_offset = *slot;
    resp.shm_size = need;
    return send_frame(fd, STATUS_OK, encode_hybrid_response(resp));
  }
  // OP_METRICS and unknown ops: not served
  return send_frame(fd, STATUS_ERR, "");
}

// --------------------------------------------------------------- ShmServer
ShmServer::ShmServer(py::object handler, const std::string& name, size_t size, int workers,
                     const std::map<uint32_t, uint32_t>& model_weights)
    : handler_(std::move(handler)), workers_(std::max(1, workers)) {
  region_ = std::make_unique<shm::Region>(shm::Region::create(name, size));
  shm::Ring<shm::ShmRequest>(region_->base() + shm::REQ_RING_OFFSET, shm::RING_CAPACITY_ARG, true);
  shm::Ring<shm::ShmResponse>(region_->base() + shm::RESP_RING_OFFSET, shm::RING_CAPACITY_ARG, true);
  const auto& h = region_->header();
  const uint64_t half = h.max_tensor_size / 2;
  result_base_ = h.tensor_pool_offset + half;
  // result slots: one sub-pool per model sized by its weight, plus the shared overflow pool
  const uint64_t bytes = h.max_tensor_size - half;
  std::vector<shm::ModelPoolSpec> specs;
  for (auto& [id, b] : shm::ModelPools::plan(bytes, {model_weights.begin(), model_weights.end()}))
    specs.push_back(shm::ModelPoolSpec{id, b, {}, {}});
  alloc_ = std::make_unique<shm::ModelPools>(result_base_, bytes, specs);
  alloc_->set_guard(region_->base());  // a result slot is reused only once its client read it
}

ShmServer::~ShmServer() {
  py::gil_scoped_release nogil;
  stop();
}

void ShmServer::start() {
  if (running_.exchange(true)) return;
  poller_ = std::thread([this] { poll_loop(); });
  for (int i = 0; i < workers_; ++i) pool_.emplace_back([this] { worker_loop(); });
}

void ShmServer::stop() {
  if (!running_.exchange(false)) return;
  if (poller_.joinable()) poller_.join();
  for (auto& t : pool_)
    if (t.joinable()) t.join();
  pool_.clear();
}

void ShmServer::poll_loop() {
  shm::Ring<shm::ShmRequest> ring(region_->base() + shm::REQ_RING_OFFSET, shm::RING_CAPACITY_ARG, false);
  int idle = 0;
  while (running_.load()) {
    auto r = ring.pop();
    if (r) {
      idle = 0;
      std::lock_guard<std::mutex> g(qmu_);
      queue_.push_back(*r);
      continue;
    }
    // short spin, then 10 us sleeps (reference polls with a 10 us sleep)
    if (++idle > 64) std::this_thread::sleep_for(std::chrono::microseconds(10));
  }
}

void ShmServer::worker_loop() {
  while (running_.load()) {
    std::optional<shm::ShmRequest> job;
    {
      std::lock_guard<std::mutex> g(qmu_);
      if (!queue_.empty()) {
        job = queue_.front();
        queue_.erase(queue_.begin());
      }
    }
    if (!job) {
      std::this_thread::sleep_for(std::chrono::microseconds(20));
      continue;
    }
    process(*job);
  }
}

void ShmServer::process(const shm::ShmRequest& req) {
  const auto t0 = std::chrono::steady_clock::now();
  shm::ShmResponse resp{};
  resp.meta.request_id = req.meta.request_id;
  std::string err;
  wire::Packet out;
  try {
    if (!region_->in_bounds(req.tensor_offset, req.tensor_size))
      throw std::out_of_range("request tensor outside the shared memory region");
    wire::Request r;
    r.input = shm::read_tensor(*region_, req.tensor_offset);
    py::gil_scoped_acquire gil;
    try {
      out = packet_from_py(
          handler_.attr("infer")(req.meta.model_id, request_to_py(r), req.meta.priority == 0 ? "latency" : "throughput"));
    } catch (py::error_already_set& e) {
      err = py_error_message(e);
    }
  } catch (const std::exception& e) {
    err = e.what();
  }
  if (err.empty()) {
    const uint64_t need = shm::tensor_bytes(out);
    auto slot = alloc_->try_allocate(req.meta.model_id, need + shm::kResultGuard, /*force=*/true);
    if (!slot) {
      exhausted_.fetch_add(1);
      err = "SHM tensor pool exhausted (required=" + std::to_string(need) + " bytes)";
    } else {
      shm::write_tensor(*region_, *slot + shm::kResultGuard, out);
      resp.result_offset = *slot + shm::kResultGuard;
      resp.result_size = need;
    }
  }
  if (!err.empty()) {
    resp.meta.status = 1;
    auto slot = alloc_->try_allocate(req.meta.model_id, 8 + err.size() + shm::kResultGuard, /*force=*/true);
    if (slot) {
      shm::write_error(*region_, *slot + shm::kResultGuard, err);
      resp.error_offset = *slot + shm::kResultGuard;
    }
  }
  resp.meta.latency_ns =
      (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count();
  shm::Ring<shm::ShmResponse> ring(region_->base() + shm::RESP_RING_OFFSET, shm::RING_CAPACITY_ARG, false);
  {
    std::lock_guard<std::mutex> g(push_mu_);
    for (int tries = 0; !ring.push(resp) && tries < 100000; ++tries) std::this_thread::sleep_for(std::chrono::microseconds(10));
  }
  const int wfd = region_->header().notify_write_fd;
  if (wfd >= 0) {
    const char one = 1;
    ssize_t n = write(wfd, &one, 1);
    (void)n;
  }
  served_.fetch_add(1);
}

}  // namespace kapsl

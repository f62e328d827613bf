// Native request servers: Unix-domain socket, TCP and shared memory.
//
// Framing and behaviour follow crates/kapsl-ipc/src/server.rs:69-676 and
// crates/kapsl-shm/src/server.rs:311-727:
//   request frame  = LE u32 model_id, u32 op_code, u32 payload_size, payload
//   response frame = LE u32 status, u32 payload_size, payload
//   OP_INFER        -> OK + bincode BinaryTensorPacket | ERR + utf8 message
//   OP_INFER_STREAM -> n x CHUNK + END; a failure before the first chunk
//                      (decode, auth, unknown model, stream start) sends only
//                      ERR; a failure mid-stream sends ERR then END
//   OP_METRICS      -> ERR with an empty payload (not served)
//   OP_HYBRID_INFER -> input tensor read from SHM at the client's offset,
//                      result written to a server-leased SHM slot, bincode
//                      HybridResponse returned
//   auth: when a token is configured, metadata.auth_token must match exactly,
//         else ERR "Unauthorized" (infer and stream ops)
// Sockets are served by native threads (one per connection); model execution
// is delegated to a Python handler object, called with the GIL held only for
// the call itself.  Every SHM offset/size from a client is bounds-checked.
#pragma once

#include "token_channel.h"
#include <pybind11/pybind11.h>

#include <atomic>
#include <memory>
#include <mutex>
#include <optional>
#include <string>
#include <thread>
#include <vector>

#include "shm.h"
#include "wire.h"

namespace kapsl {

namespace py = pybind11;

py::dict request_to_py(const wire::Request& r);
wire::Packet packet_from_py(const py::handle& obj);
py::tuple packet_to_py(const wire::Packet& p);

class WireServer {
 public:
  // handler: object with infer(model_id, request_dict, priority) -> (shape, dtype, data)
  //          and infer_stream(model_id, request_dict) -> iterator of (shape, dtype, data)
  WireServer(py::object handler, std::optional<std::string> auth_token);
  ~WireServer();
  void listen_unix(const std::string& path);
  int listen_tcp(const std::string& host, int port);  // returns the bound port
  void attach_shm(const std::string& shm_name);       // enables OP_HYBRID_INFER
  void start();
  void stop();
  bool running() const { return running_.load(); }
  uint64_t requests_served() const { return served_.load(); }

 private:
  void accept_loop(int lfd);
  void serve_connection(int fd);
  bool handle_frame(int fd, uint32_t model_id, uint32_t op, const std::string& payload);
  bool send_frame(int fd, uint32_t status, const std::string& payload);
  bool stream_channel(int fd, TokenChannel& ch);
  std::optional<std::string> check_auth(const wire::Request& r) const;

  py::object handler_;
  std::optional<std::string> token_;
  std::vector<int> listen_fds_;
  std::string unix_path_;
  std::vector<std::thread> threads_;
  std::mutex conn_mu_;
  std::vector<int> conn_fds_;
  struct Conn {
    std::thread t;
    std::shared_ptr<std::atomic<bool>> done;
  };
  std::vector<Conn> conns_;  // finished ones are joined by the accept loop
  std::atomic<bool> running_{false};
  std::atomic<uint64_t> served_{0};
  std::unique_ptr<shm::Region> hybrid_region_;
  std::unique_ptr<shm::TieredAllocator> hybrid_alloc_;
};

class ShmServer {
 public:
  ShmServer(py::object handler, const std::string& name, size_t size, int workers,
            const std::map<uint32_t, uint32_t>& model_weights = {});
  ~ShmServer();
  void start();
  void stop();
  uint64_t requests_served() const { return served_.load(); }
  size_t pool_in_use() const { return alloc_ ? alloc_->total_usage().in_use : 0; }
  double pool_oldest_lease_ms() const { return alloc_ ? alloc_->total_usage().oldest_lease_ms : 0.0; }
  const shm::ModelPools* pools() const { return alloc_.get(); }
  uint64_t pool_exhausted() const { return exhausted_.load(); }
  uint64_t result_pool_base() const { return result_base_; }

 private:
  void poll_loop();
  void worker_loop();
  void process(const shm::ShmRequest& req);

  py::object handler_;
  std::unique_ptr<shm::Region> region_;
  std::unique_ptr<shm::ModelPools> alloc_;
  uint64_t result_base_ = 0;
  int workers_;
  std::atomic<bool> running_{false};
  std::atomic<uint64_t> served_{0};
  std::atomic<uint64_t> exhausted_{0};
  std::thread poller_;
  std::vector<std::thread> pool_;
  std::mutex qmu_;
  std::vector<shm::ShmRequest> queue_;
  std::mutex push_mu_;
};

}  // namespace kapsl

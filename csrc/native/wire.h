// bincode-1.3 (legacy config) codec for the kapsl wire protocol.
//
// Encoding rules (bincode::serialize / deserialize free functions): fixed-width
// little-endian integers, u64 length prefixes for Vec / String / bytes,
// Option = 1-byte tag (0/1) then the value, fixed arrays without a length,
// structs as their fields in declaration order, bool = 1 byte.
//
// Types and field orders follow crates/kapsl-engine-api/src/lib.rs
// (BinaryTensorPacket 272-339, RequestMetadata 462-492, InferenceRequest
// 521-532), crates/kapsl-transport/src/lib.rs:37-97 (24-byte request /
// response metadata) and crates/kapsl-ipc/src/protocol.rs (frames, hybrid
// messages, op and status codes).
#pragma once

#include <stdint.h>

#include <optional>
#include <stdexcept>
#include <string>
#include <vector>

namespace kapsl {
namespace wire {

constexpr uint32_t OP_INFER = 1;
constexpr uint32_t OP_INFER_STREAM = 2;
constexpr uint32_t OP_METRICS = 3;
constexpr uint32_t OP_HYBRID_INFER = 4;
constexpr uint32_t STATUS_OK = 0;
constexpr uint32_t STATUS_ERR = 1;
constexpr uint32_t STATUS_STREAM_CHUNK = 2;
constexpr uint32_t STATUS_STREAM_END = 3;

struct DecodeError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

class Writer {
 public:
  std::string buf;
  void u8(uint8_t v) { buf.push_back((char)v); }
  void boolean(bool v) { u8(v ? 1 : 0); }
  void u32(uint32_t v) { raw(&v, 4); }
  void u64(uint64_t v) { raw(&v, 8); }
  void i64(int64_t v) { raw(&v, 8); }
  void f32(float v) { raw(&v, 4); }
  void bytes(const std::string& s) {
    u64(s.size());
    buf.append(s);
  }
  void str(const std::string& s) { bytes(s); }
  void raw(const void* p, size_t n) { buf.append(reinterpret_cast<const char*>(p), n); }
};

class Reader {
 public:
  Reader(const uint8_t* p, size_t n) : p_(p), n_(n) {}
  explicit Reader(const std::string& s) : p_(reinterpret_cast<const uint8_t*>(s.data())), n_(s.size()) {}
  uint8_t u8() {
    need(1);
    return p_[off_++];
  }
  bool boolean() {
    uint8_t v = u8();
    if (v > 1) throw DecodeError("invalid bool byte");
    return v == 1;
  }
  bool tag() {
    uint8_t v = u8();
    if (v > 1) throw DecodeError("invalid Option tag");
    return v == 1;
  }
  uint32_t u32() { return get<uint32_t>(); }
  uint64_t u64() { return get<uint64_t>(); }
  int64_t i64() { return get<int64_t>(); }
  float f32() { return get<float>(); }
  std::string bytes() {
    uint64_t n = u64();
    need(n);
    std::string s(reinterpret_cast<const char*>(p_ + off_), (size_t)n);
    off_ += n;
    return s;
  }
  std::string str();  // bytes + UTF-8 validation
  size_t remaining() const { return n_ - off_; }
  size_t offset() const { return off_; }

 private:
  template <class T>
  T get() {
    need(sizeof(T));
    T v;
    memcpy_(&v, p_ + off_, sizeof(T));
    off_ += sizeof(T);
    return v;
  }
  static void memcpy_(void* d, const void* s, size_t n);
  void need(uint64_t n) {
    if (n > n_ - off_) throw DecodeError("unexpected end of payload");
  }
  const uint8_t* p_;
  size_t n_;
  size_t off_ = 0;
};

// TensorDtype is carried as its string name; parse accepts the aliases.
bool dtype_parse(const std::string& s, std::string* canonical, int* itemsize);

struct Packet {
  std::vector<int64_t> shape;
  std::string dtype;  // canonical name
  std::string data;
};

struct NamedTensor {
  std::string name;
  Packet tensor;
};

struct Metadata {
  std::optional<std::string> request_id;
  std::optional<uint64_t> timeout_ms;
  std::optional<uint8_t> priority;
  std::optional<bool> force_cpu;
  std::optional<std::string> model_version;
  std::optional<std::string> auth_token;  // omitted on the wire when None
  std::optional<uint32_t> max_new_tokens;
  std::optional<float> temperature;
  std::optional<float> top_p;
  std::optional<uint32_t> top_k;
  std::optional<float> repetition_penalty;
  std::optional<uint64_t> seed;
  std::optional<std::vector<uint32_t>> stop_token_ids;
};

struct Request {
  Packet input;
  std::vector<NamedTensor> additional_inputs;
  std::optional<std::string> session_id;
  std::optional<Metadata> metadata;
};

// 24-byte #[repr(C)] structs shared by the SHM rings and hybrid messages.
struct TransportRequestMeta {
  uint64_t request_id = 0;
  uint32_t model_id = 0;
  uint8_t priority = 0;
  uint8_t force_cpu = 0;
  uint8_t padding[2] = {0, 0};
  uint64_t timestamp_ns = 0;
};
struct TransportResponseMeta {
  uint64_t request_id = 0;
  uint8_t status = 0;
  uint8_t padding[7] = {0, 0, 0, 0, 0, 0, 0};
  uint64_t latency_ns = 0;
};
static_assert(sizeof(TransportRequestMeta) == 24, "request metadata is 24 bytes");
static_assert(sizeof(TransportResponseMeta) == 24, "response metadata is 24 bytes");

struct HybridRequest {
  TransportRequestMeta meta;
  uint64_t shm_offset = 0;
  uint64_t shm_size = 0;
};
struct HybridResponse {
  TransportResponseMeta meta;
  uint64_t shm_offset = 0;
  uint64_t shm_size = 0;
};

void encode_packet(Writer& w, const Packet& p);
Packet decode_packet(Reader& r);
std::string encode_packet(const Packet& p);
Packet decode_packet(const std::string& s);

void encode_metadata(Writer& w, const Metadata& m);
std::string encode_request(const Request& req);
// Positional decode with the full field layout; on failure retries with the
// auth_token field omitted, then the legacy {input, additional_inputs,
// session_id} layout (crates/kapsl-ipc/src/server.rs:27-67).
Request decode_request(const std::string& payload);

std::string encode_hybrid_request(const HybridRequest& h);
HybridRequest decode_hybrid_request(const std::string& s);
std::string encode_hybrid_response(const HybridResponse& h);
HybridResponse decode_hybrid_response(const std::string& s);

// Frame headers (raw little-endian u32s).
std::string request_header(uint32_t model_id, uint32_t op, uint32_t size);
std::string response_header(uint32_t status, uint32_t size);

// Validates shape (dims > 0) and byte length against dtype; returns "" if ok,
// else the reference's InvalidInput message.
std::string validate_packet(const Packet& p);

}  // namespace wire
}  // namespace kapsl

#include "wire.h"

#include <cstring>

namespace kapsl {
namespace wire {

void Reader::memcpy_(void* d, const void* s, size_t n) { std::memcpy(d, s, n); }

static bool valid_utf8(const std::string& s) {
  size_t i = 0, n = s.size();
  const unsigned char* p = reinterpret_cast<const unsigned char*>(s.data());
  while (i < n) {
    unsigned c = p[i];
    size_t len = c < 0x80 ? 1 : (c >> 5) == 0x6 ? 2 : (c >> 4) == 0xE ? 3 : (c >> 3) == 0x1E ? 4 : 0;
    if (len == 0 || i + len > n) return false;
    for (size_t k = 1; k < len; ++k)
      if ((p[i + k] & 0xC0) != 0x80) return false;
    i += len;
  }
  return true;
}

std::string Reader::str() {
  std::string s = bytes();
  if (!valid_utf8(s)) throw DecodeError("invalid utf-8 in string");
  return s;
}

bool dtype_parse(const std::string& s, std::string* canonical, int* itemsize) {
  std::string k;
  k.reserve(s.size());
  for (char c : s) k.push_back((char)std::tolower((unsigned char)c));
  struct E {
    const char* a;
    const char* c;
    int sz;
  };
  static const E table[] = {{"float32", "float32", 4}, {"fp32", "float32", 4}, {"float64", "float64", 8},
                            {"fp64", "float64", 8},    {"float16", "float16", 2}, {"fp16", "float16", 2},
                            {"int32", "int32", 4},     {"i32", "int32", 4},      {"int64", "int64", 8},
                            {"i64", "int64", 8},       {"uint8", "uint8", 1},    {"u8", "uint8", 1},
                            {"string", "string", 1},   {"utf8", "string", 1}};
  for (const E& e : table)
    if (k == e.a) {
      if (canonical) *canonical = e.c;
      if (itemsize) *itemsize = e.sz;
      return true;
    }
  return false;
}

static const char kB64[] = "ABCDEFGHIJKLMNOPQRSTUVWXYZabcdefghijklmnopqrstuvwxyz0123456789+/";

static std::string b64_decode(const std::string& in) {
  int val[256];
  for (int i = 0; i < 256; ++i) val[i] = -1;
  for (int i = 0; i < 64; ++i) val[(unsigned char)kB64[i]] = i;
  std::string out;
  int buf = 0, bits = 0;
  size_t pad = 0;
  for (unsigned char c : in) {
    if (c == '=') {
      ++pad;
      continue;
    }
    if (pad) throw DecodeError("invalid base64 padding");
    if (val[c] < 0) throw DecodeError("invalid base64 symbol");
    buf = (buf << 6) | val[c];
    bits += 6;
    if (bits >= 8) {
      bits -= 8;
      out.push_back((char)((buf >> bits) & 0xFF));
    }
  }
  if ((in.size() % 4) != 0) throw DecodeError("invalid base64 length");
  return out;
}

void encode_packet(Writer& w, const Packet& p) {
  w.u64(p.shape.size());
  for (int64_t d : p.shape) w.i64(d);
  w.str(p.dtype);
  w.u8(1);  // data: Some
  w.bytes(p.data);
  w.u8(0);  // data_base64: None
}

Packet decode_packet(Reader& r) {
  Packet p;
  uint64_t nd = r.u64();
  if (nd > (1u << 20)) throw DecodeError("shape too long");
  p.shape.resize(nd);
  for (uint64_t i = 0; i < nd; ++i) p.shape[i] = r.i64();
  std::string dt = r.str();
  int sz = 0;
  if (!dtype_parse(dt, &p.dtype, &sz)) throw DecodeError("Unsupported dtype: " + dt);
  bool has_data = r.tag();
  std::string data;
  if (has_data) data = r.bytes();
  bool has_b64 = r.tag();
  std::string b64;
  if (has_b64) b64 = r.str();
  if (has_data && has_b64) throw DecodeError("binary tensor payload must include only one of `data` or `data_base64`");
  if (!has_data && !has_b64) throw DecodeError("binary tensor payload must include `data` or `data_base64`");
  p.data = has_data ? std::move(data) : b64_decode(b64);
  return p;
}

std::string encode_packet(const Packet& p) {
  Writer w;
  encode_packet(w, p);
  return w.buf;
}

Packet decode_packet(const std::string& s) {
  Reader r(s);
  return decode_packet(r);
}

template <class T, class F>
static void opt(Writer& w, const std::optional<T>& v, F f) {
  if (v.has_value()) {
    w.u8(1);
    f(*v);
  } else {
    w.u8(0);
  }
}

void encode_metadata(Writer& w, const Metadata& m) {
  opt(w, m.request_id, [&](const std::string& s) { w.str(s); });
  opt(w, m.timeout_ms, [&](uint64_t v) { w.u64(v); });
  opt(w, m.priority, [&](uint8_t v) { w.u8(v); });
  opt(w, m.force_cpu, [&](bool v) { w.boolean(v); });
  opt(w, m.model_version, [&](const std::string& s) { w.str(s); });
  if (m.auth_token.has_value()) {  // skip_serializing_if = "Option::is_none"
    w.u8(1);
    w.str(*m.auth_token);
  }
  opt(w, m.max_new_tokens, [&](uint32_t v) { w.u32(v); });
  opt(w, m.temperature, [&](float v) { w.f32(v); });
  opt(w, m.top_p, [&](float v) { w.f32(v); });
  opt(w, m.top_k, [&](uint32_t v) { w.u32(v); });
  opt(w, m.repetition_penalty, [&](float v) { w.f32(v); });
  opt(w, m.seed, [&](uint64_t v) { w.u64(v); });
  opt(w, m.stop_token_ids, [&](const std::vector<uint32_t>& ids) {
    w.u64(ids.size());
    for (uint32_t x : ids) w.u32(x);
  });
}

static Metadata decode_metadata(Reader& r, bool with_auth) {
  Metadata m;
  if (r.tag()) m.request_id = r.str();
  if (r.tag()) m.timeout_ms = r.u64();
  if (r.tag()) m.priority = r.u8();
  if (r.tag()) m.force_cpu = r.boolean();
  if (r.tag()) m.model_version = r.str();
  if (with_auth && r.tag()) m.auth_token = r.str();
  if (r.tag()) m.max_new_tokens = r.u32();
  if (r.tag()) m.temperature = r.f32();
  if (r.tag()) m.top_p = r.f32();
  if (r.tag()) m.top_k = r.u32();
  if (r.tag()) m.repetition_penalty = r.f32();
  if (r.tag()) m.seed = r.u64();
  if (r.tag()) {
    uint64_t n = r.u64();
    if (n > (1u << 24)) throw DecodeError("stop_token_ids too long");
    std::vector<uint32_t> ids(n);
    for (uint64_t i = 0; i < n; ++i) ids[i] = r.u32();
    m.stop_token_ids = std::move(ids);
  }
  return m;
}

std::string encode_request(const Request& req) {
  Writer w;
  encode_packet(w, req.input);
  w.u64(req.additional_inputs.size());
  for (const auto& nt : req.additional_inputs) {
    w.str(nt.name);
    encode_packet(w, nt.tensor);
  }
  opt(w, req.session_id, [&](const std::string& s) { w.str(s); });
  opt(w, req.metadata, [&](const Metadata& m) { encode_metadata(w, m); });
  return w.buf;
}

static Request decode_request_layout(const std::string& payload, int layout, bool exact) {
  // layout 0: full; 1: metadata without auth_token; 2: legacy (no metadata).
  // exact: the layout must consume the whole payload.
  Reader r(payload);
  Request req;
  req.input = decode_packet(r);
  uint64_t n = r.u64();
  if (n > (1u << 20)) throw DecodeError("too many additional inputs");
  for (uint64_t i = 0; i < n; ++i) {
    NamedTensor nt;
    nt.name = r.str();
    nt.tensor = decode_packet(r);
    req.additional_inputs.push_back(std::move(nt));
  }
  if (r.tag()) req.session_id = r.str();
  if (layout != 2) {
    if (r.tag()) req.metadata = decode_metadata(r, layout == 0);
  }
  if (exact && r.remaining() != 0) throw DecodeError("trailing bytes after InferenceRequest");
  return req;
}

// Metadata serialised without its auth_token (the field is skipped when None) is
// one Option tag shorter, and the full layout can read such a payload without an
// error while misplacing every later field (a seed read as repetition_penalty, the
// seed itself dropped).  So the layouts are first tried in order where they must
// consume the payload exactly, then in the same order as a plain prefix parse
// (legacy payloads with trailing bytes).
Request decode_request(const std::string& payload) {
  std::string first;
  for (bool exact : {true, false}) {
    for (int layout = 0; layout < 3; ++layout) {
      try {
        return decode_request_layout(payload, layout, exact);
      } catch (const DecodeError& e) {
        if (first.empty()) first = e.what();
      }
    }
  }
  throw DecodeError(std::string("failed to decode InferenceRequest: ") + first);
}

static void enc_tmeta(Writer& w, const TransportRequestMeta& m) {
  w.u64(m.request_id);
  w.u32(m.model_id);
  w.u8(m.priority);
  w.u8(m.force_cpu);
  w.u8(m.padding[0]);
  w.u8(m.padding[1]);
  w.u64(m.timestamp_ns);
}
static TransportRequestMeta dec_tmeta(Reader& r) {
  TransportRequestMeta m;
  m.request_id = r.u64();
  m.model_id = r.u32();
  m.priority = r.u8();
  m.force_cpu = r.boolean() ? 1 : 0;
  m.padding[0] = r.u8();
  m.padding[1] = r.u8();
  m.timestamp_ns = r.u64();
  return m;
}
static void enc_rmeta(Writer& w, const TransportResponseMeta& m) {
  w.u64(m.request_id);
  w.u8(m.status);
  for (int i = 0; i < 7; ++i) w.u8(m.padding[i]);
  w.u64(m.latency_ns);
}
static TransportResponseMeta dec_rmeta(Reader& r) {
  TransportResponseMeta m;
  m.request_id = r.u64();
  m.status = r.u8();
  for (int i = 0; i < 7; ++i) m.padding[i] = r.u8();
  m.latency_ns = r.u64();
  return m;
}

std::string encode_hybrid_request(const HybridRequest& h) {
  Writer w;
  enc_tmeta(w, h.meta);
  w.u64(h.shm_offset);
  w.u64(h.shm_size);
  return w.buf;
}
HybridRequest decode_hybrid_request(const std::string& s) {
  Reader r(s);
  HybridRequest h;
  h.meta = dec_tmeta(r);
  h.shm_offset = r.u64();
  h.shm_size = r.u64();
  return h;
}
std::string encode_hybrid_response(const HybridResponse& h) {
  Writer w;
  enc_rmeta(w, h.meta);
  w.u64(h.shm_offset);
  w.u64(h.shm_size);
  return w.buf;
}
HybridResponse decode_hybrid_response(const std::string& s) {
  Reader r(s);
  HybridResponse h;
  h.meta = dec_rmeta(r);
  h.shm_offset = r.u64();
  h.shm_size = r.u64();
  return h;
}

std::string request_header(uint32_t model_id, uint32_t op, uint32_t size) {
  Writer w;
  w.u32(model_id);
  w.u32(op);
  w.u32(size);
  return w.buf;
}
std::string response_header(uint32_t status, uint32_t size) {
  Writer w;
  w.u32(status);
  w.u32(size);
  return w.buf;
}

std::string validate_packet(const Packet& p) {
  uint64_t elems = 1;
  for (int64_t d : p.shape) {
    if (d <= 0) return "Invalid shape dimension: " + std::to_string(d);
    if (elems > UINT64_MAX / (uint64_t)d) return "Shape multiplication overflow";
    elems *= (uint64_t)d;
  }
  int sz = 1;
  std::string canon;
  if (!dtype_parse(p.dtype, &canon, &sz)) return "Unsupported dtype: " + p.dtype;
  const uint64_t expected = elems * (uint64_t)sz;
  if (p.data.size() != expected)
    return "Data length mismatch: expected " + std::to_string(expected) + " bytes (" + std::to_string(elems) + " " +
           canon + " values) but got " + std::to_string(p.data.size()) + " bytes";
  return "";
}

}  // namespace wire
}  // namespace kapsl

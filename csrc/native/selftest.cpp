// Standalone self-test of the C++ runtime pieces that run without Python: the
// SHM region and MPMC rings, the slot / tiered / per-model allocators, the
// cross-process lease words, the paged-KV block allocator, the bincode codec and
// the CPU kernels' thread pool.  Built with -fsanitize=thread and with
// -fsanitize=address,undefined so races and memory errors in this code show up
// on the host (device code has its own bounds checks).
//
//   g++ -std=c++17 -O1 -g -fsanitize=thread selftest.cpp shm.cpp wire.cpp \
//       block_alloc.cpp cpu_kernels.cpp -I. -pthread -lrt -o selftest && ./selftest
//
// Exit status 0 means every check passed; each failed check prints one line.
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <set>
#include <string>
#include <thread>
#include <vector>

#include "block_alloc.h"
#include "cpu_kernels.h"
#include "hnsw.h"
#include "shm.h"
#include "text_index.h"
#include "token_channel.h"
#include "wasm.h"
#include "wire.h"

using namespace kapsl;

static int g_failures = 0;
#define CHECK(cond, ...)                                   \
  do {                                                     \
    if (!(cond)) {                                         \
      ++g_failures;                                        \
      std::fprintf(stderr, "FAIL %s:%d: ", __FILE__, __LINE__); \
      std::fprintf(stderr, __VA_ARGS__);                   \
      std::fprintf(stderr, "\n");                          \
    }                                                      \
  } while (0)

static std::string region_name(const char* tag) {
  return std::string("kapsl-selftest-") + tag + "-" + std::to_string(getpid());
}

// Producers and consumers hammer one ring; every item arrives exactly once.
static void test_ring_mpmc() {
  shm::Region r = shm::Region::create(region_name("ring"), 1 << 20);
  shm::Ring<shm::ShmRequest> init(r.base() + shm::REQ_RING_OFFSET, shm::RING_CAPACITY_ARG, true);
  constexpr int P = 4, C = 4, N = 5000;
  std::vector<std::atomic<uint8_t>> seen(P * N);
  for (auto& s : seen) s.store(0);
  std::atomic<int> got{0};
  std::vector<std::thread> ts;
  for (int p = 0; p < P; ++p)
    ts.emplace_back([&, p] {
      shm::Ring<shm::ShmRequest> q(r.base() + shm::REQ_RING_OFFSET, shm::RING_CAPACITY_ARG, false);
      for (int i = 0; i < N; ++i) {
        shm::ShmRequest it{};
        it.meta.request_id = (uint64_t)p * N + i;
        it.tensor_offset = it.meta.request_id * 7;
        while (!q.push(it)) std::this_thread::yield();
      }
    });
  for (int c = 0; c < C; ++c)
    ts.emplace_back([&] {
      shm::Ring<shm::ShmRequest> q(r.base() + shm::REQ_RING_OFFSET, shm::RING_CAPACITY_ARG, false);
      const auto t0 = std::chrono::steady_clock::now();
      while (got.load() < P * N && std::chrono::steady_clock::now() - t0 < std::chrono::seconds(60)) {
        auto it = q.pop();
        if (!it) {
          std::this_thread::yield();
          continue;
        }
        const uint64_t id = it->meta.request_id;
        CHECK(id < (uint64_t)P * N && it->tensor_offset == id * 7, "ring: corrupt item %llu", (unsigned long long)id);
        if (id < (uint64_t)P * N) CHECK(seen[id].fetch_add(1) == 0, "ring: item %llu twice", (unsigned long long)id);
        got.fetch_add(1);
      }
    });
  for (auto& t : ts) t.join();
  CHECK(got.load() == P * N, "ring: %d of %d items arrived", got.load(), P * N);
}

// The SHM client pattern: clients share one response ring, pop whatever is at
// the tail and push back responses addressed to someone else.  Every client
// must receive all of its own responses.
static void test_ring_repush() {
  shm::Region r = shm::Region::create(region_name("repush"), 1 << 20);
  shm::Ring<shm::ShmResponse> init(r.base() + shm::RESP_RING_OFFSET, shm::RING_CAPACITY_ARG, true);
  constexpr int K = 4, N = 500;
  std::atomic<int> done{0};
  std::vector<std::thread> ts;
  ts.emplace_back([&] {  // the server: responses for every client, interleaved
    shm::Ring<shm::ShmResponse> q(r.base() + shm::RESP_RING_OFFSET, shm::RING_CAPACITY_ARG, false);
    for (int i = 0; i < N; ++i)
      for (int k = 0; k < K; ++k) {
        shm::ShmResponse it{};
        it.meta.request_id = ((uint64_t)k << 32) | (uint64_t)i;
        // keep room for the clients' pushes back (a full ring would leave every
        // client holding a popped response it cannot return)
        while (q.len() > 64) std::this_thread::yield();
        while (!q.push(it)) std::this_thread::yield();
      }
  });
  for (int k = 0; k < K; ++k)
    ts.emplace_back([&, k] {
      shm::Ring<shm::ShmResponse> q(r.base() + shm::RESP_RING_OFFSET, shm::RING_CAPACITY_ARG, false);
      std::vector<uint8_t> mine(N, 0);
      int have = 0;
      const auto t0 = std::chrono::steady_clock::now();
      while (have < N && std::chrono::steady_clock::now() - t0 < std::chrono::seconds(60)) {
        auto it = q.pop();
        if (!it) {
          std::this_thread::yield();
          continue;
        }
        const uint64_t owner = it->meta.request_id >> 32, idx = it->meta.request_id & 0xffffffffu;
        if ((int)owner != k) {
          while (!q.push(*it)) std::this_thread::yield();
          continue;
        }
        CHECK(idx < (uint64_t)N && !mine[idx], "repush: client %d got %llu twice", k, (unsigned long long)idx);
        if (idx < (uint64_t)N) mine[idx] = 1;
        ++have;
      }
      CHECK(have == N, "repush: client %d got %d of %d responses", k, have, N);
      done.fetch_add(1);
    });
  for (auto& t : ts) t.join();
}

// Concurrent allocate / release on the per-model pools: no offset is ever
// handed to two holders at once.
static void test_model_pools() {
  const uint64_t MiB = 1 << 20;
  auto plan = shm::ModelPools::plan(64 * MiB, {{1, 3}, {2, 1}});
  std::vector<shm::ModelPoolSpec> specs;
  for (auto& [id, b] : plan) specs.push_back({id, b, {256 << 10, MiB}, {3, 1}});
  shm::ModelPools pools(4096, 64 * MiB, specs, 60.0);
  std::mutex mu;
  std::set<uint64_t> held;
  std::vector<std::thread> ts;
  for (int t = 0; t < 6; ++t)
    ts.emplace_back([&, t] {
      std::mt19937 rng(t);
      std::vector<uint64_t> mine;
      for (int i = 0; i < 4000; ++i) {
        if (mine.size() < 8 && rng() % 3) {
          const uint32_t model = rng() % 4;  // 0 and 3 have no pool of their own
          const uint64_t size = 1 + rng() % (MiB - 1);
          if (auto o = pools.try_allocate(model, size)) {
            std::lock_guard<std::mutex> g(mu);
            CHECK(held.insert(*o).second, "pools: offset %llu handed out twice", (unsigned long long)*o);
            mine.push_back(*o);
          }
        } else if (!mine.empty()) {
          const uint64_t o = mine.back();
          mine.pop_back();
          {
            std::lock_guard<std::mutex> g(mu);
            held.erase(o);
          }
          CHECK(pools.release(o), "pools: release of %llu failed", (unsigned long long)o);
        }
      }
      for (uint64_t o : mine) {
        {
          std::lock_guard<std::mutex> g(mu);
          held.erase(o);
        }
        pools.release(o);
      }
    });
  for (auto& t : ts) t.join();
  CHECK(pools.total_usage().in_use == 0, "pools: %zu slots still leased", pools.total_usage().in_use);
}

// Two lease tables over one region (two client processes): exclusive slots.
static void test_shared_leases() {
  shm::Region r = shm::Region::create(region_name("lease"), 8 << 20);
  const uint64_t base = shm::TENSOR_POOL_OFFSET, bytes = r.size() - base;
  std::mutex mu;
  std::set<uint64_t> held;
  std::vector<std::thread> ts;
  for (int t = 0; t < 4; ++t)
    ts.emplace_back([&, t] {
      shm::SharedLeases leases(r, base, bytes, 60.0);
      std::mt19937 rng(100 + t);
      for (int i = 0; i < 3000; ++i) {
        if (auto o = leases.try_allocate(1 + rng() % (200 << 10))) {
          {
            std::lock_guard<std::mutex> g(mu);
            CHECK(held.insert(*o).second, "leases: offset %llu leased twice", (unsigned long long)*o);
          }
          std::this_thread::yield();
          {
            std::lock_guard<std::mutex> g(mu);
            held.erase(*o);
          }
          CHECK(leases.release(*o), "leases: release failed");
        }
      }
    });
  for (auto& t : ts) t.join();
}

// Random allocate / free / prefix traffic on the block allocator; the free
// count always balances.
static void test_block_allocator() {
  for (const char* ev : {"lru", "fifo"}) {
    BlockAllocator a(64, 4, true, ev);
    std::mt19937 rng(7);
    std::vector<std::pair<std::vector<int32_t>, std::vector<int64_t>>> held;
    for (int step = 0; step < 20000; ++step) {
      const int op = rng() % 10;
      if (op < 4) {
        const int n = 1 + rng() % 5;
        try {
          auto b = a.allocate(n);
          std::vector<int32_t> toks(4 * n);
          for (auto& x : toks) x = rng() % 3;
          held.push_back({toks, b});
        } catch (const OutOfBlocksError&) {
        }
      } else if (op < 6 && !held.empty()) {
        auto& h = held[rng() % held.size()];
        a.commit_prefix(h.first, h.second, (int)(rng() % 4));
      } else if (op < 8 && !held.empty()) {
        const size_t i = rng() % held.size();
        a.free(held[i].second);
        held.erase(held.begin() + i);
      } else {
        std::vector<int32_t> toks(1 + rng() % 20);
        for (auto& x : toks) x = rng() % 3;
        auto m = a.match_prefix(toks);
        if (!m.empty()) held.push_back({std::vector<int32_t>(toks.begin(), toks.begin() + 4 * m.size()), m});
      }
      int64_t used = 0;
      for (auto& h : held) used += (int64_t)h.second.size();
      CHECK(a.num_used() <= used, "blocks: %lld used but %lld held", (long long)a.num_used(), (long long)used);
    }
    for (auto& h : held) a.free(h.second);
    CHECK(a.num_free() == 64, "blocks: %lld free after releasing everything", (long long)a.num_free());
  }
}

// Round trips, then every truncated prefix of an encoded request must be
// rejected without reading past the payload.
static void test_wire() {
  std::mt19937 rng(3);
  for (int i = 0; i < 200; ++i) {
    wire::Request req;
    req.input.shape = {1 + (int64_t)(rng() % 4), 1 + (int64_t)(rng() % 5)};
    req.input.dtype = "float32";
    req.input.data.assign(req.input.shape[0] * req.input.shape[1] * 4, (char)(rng() & 0xff));
    if (rng() % 2) req.session_id = "s" + std::to_string(i);
    if (rng() % 2) {
      wire::Metadata m;
      m.request_id = "r" + std::to_string(i);
      if (rng() % 2) m.auth_token = "tok";
      if (rng() % 2) m.temperature = 0.5f;
      if (rng() % 2) m.stop_token_ids = std::vector<uint32_t>{1, 2, 3};
      req.metadata = m;
    }
    const std::string enc = wire::encode_request(req);
    wire::Request back = wire::decode_request(enc);
    CHECK(back.input.data == req.input.data && back.input.shape == req.input.shape &&
              back.session_id == req.session_id,
          "wire: round trip %d", i);
    for (size_t n = 0; n < enc.size(); n += 1 + enc.size() / 64) {
      try {
        wire::decode_request(enc.substr(0, n));
      } catch (const std::exception&) {
      }
    }
  }
}

// The CPU kernels' worker pool from several caller threads at once.
static void test_cpu_pool() {
  const int64_t rows = 257, d = 300;
  std::vector<std::thread> ts;
  for (int t = 0; t < 3; ++t)
    ts.emplace_back([&, t] {
      std::mt19937 rng(t);
      std::uniform_real_distribution<float> U(-1, 1);
      std::vector<float> x(rows * d), w(d), out(rows * d);
      for (auto& v : x) v = U(rng);
      for (auto& v : w) v = U(rng);
      cpu::rmsnorm(x.data(), w.data(), out.data(), rows, d, 1e-5f);
      for (int64_t r = 0; r < rows; r += 37) {
        double ss = 0;
        for (int64_t j = 0; j < d; ++j) ss += (double)x[r * d + j] * x[r * d + j];
        const double inv = 1.0 / std::sqrt(ss / d + 1e-5);
        for (int64_t j = 0; j < d; j += 29)
          CHECK(std::fabs(out[r * d + j] - x[r * d + j] * inv * w[j]) < 1e-4, "cpu pool: rmsnorm row %lld",
                (long long)r);
      }
    });
  for (auto& t : ts) t.join();
  // Q4_K: the int8-activation kernel against the fp32 one on random blocks
  // (d and dmin kept small and finite: f16 0x1400 = 2^-10, 0x1000 = 2^-11)
  const int64_t N = 33, K = 512, T = 5;
  std::mt19937 rng(11);
  std::vector<uint8_t> wq(N * (K / 256) * 144);
  for (auto& b : wq) b = (uint8_t)rng();
  for (int64_t blk = 0; blk < N * (K / 256); ++blk) {
    wq[blk * 144 + 0] = 0x00, wq[blk * 144 + 1] = 0x14;
    wq[blk * 144 + 2] = 0x00, wq[blk * 144 + 3] = 0x10;
  }
  std::uniform_real_distribution<float> U(-1, 1);
  std::vector<float> x(T * K), y0(T * N), y1(T * N);
  for (auto& v : x) v = U(rng);
  cpu::q4k_matmul(x.data(), wq.data(), y0.data(), T, N, K);
  cpu::q4k_matmul_q8(x.data(), wq.data(), y1.data(), T, N, K);
  float amax = 0.f, err = 0.f;
  for (int64_t i = 0; i < T * N; ++i) {
    amax = std::max(amax, std::fabs(y0[i]));
    err = std::max(err, std::fabs(y0[i] - y1[i]));
  }
  CHECK(err <= 0.02f * amax, "q4k int8 kernel: error %g of %g", err, amax);
  // Q6_K: the int8 kernel against dequantized rows (d = f16 0x1000 = 2^-11)
  std::vector<uint8_t> w6(N * (K / 256) * 210);
  for (auto& b : w6) b = (uint8_t)rng();
  for (int64_t blk = 0; blk < N * (K / 256); ++blk) w6[blk * 210 + 208] = 0x00, w6[blk * 210 + 209] = 0x10;
  std::vector<float> deq(N * K);
  cpu::q6k_dequant_rows(w6.data(), deq.data(), 0, N, K);
  cpu::q6k_matmul_q8(x.data(), w6.data(), y1.data(), T, N, K);
  amax = err = 0.f;
  for (int64_t t = 0; t < T; ++t)
    for (int64_t n = 0; n < N; ++n) {
      float ref = 0.f;
      for (int64_t k = 0; k < K; ++k) ref += x[t * K + k] * deq[n * K + k];
      amax = std::max(amax, std::fabs(ref));
      err = std::max(err, std::fabs(ref - y1[t * N + n]));
    }
  CHECK(err <= 0.02f * amax, "q6k int8 kernel: error %g of %g", err, amax);
  // Q8_0: the int8 kernel against dequantized rows (d = 2^-11)
  std::vector<uint8_t> w8(N * (K / 32) * 34);
  for (auto& b : w8) b = (uint8_t)rng();
  for (int64_t blk = 0; blk < N * (K / 32); ++blk) w8[blk * 34] = 0x00, w8[blk * 34 + 1] = 0x10;
  cpu::q80_dequant_rows(w8.data(), deq.data(), 0, N, K);
  cpu::q80_matmul_q8(x.data(), w8.data(), y1.data(), T, N, K);
  amax = err = 0.f;
  for (int64_t t = 0; t < T; ++t)
    for (int64_t n = 0; n < N; ++n) {
      float ref = 0.f;
      for (int64_t k = 0; k < K; ++k) ref += x[t * K + k] * deq[n * K + k];
      amax = std::max(amax, std::fabs(ref));
      err = std::max(err, std::fabs(ref - y1[t * N + n]));
    }
  CHECK(err <= 0.02f * amax, "q8_0 int8 kernel: error %g of %g", err, amax);
}

// A module with recursion, br_table, bulk memory, a mutable global, memory.grow
// and call_indirect (exports fib, switch, bulk, dispatch); then random byte
// flips of it, each of which must load-fail, trap or run, never corrupt memory.
static const char* kModuleHex =
    "0061736d01000000011c0560017e017e60017f017f6000017f60027f7f017f60037f7f7f017f03060500010203040404"
    "017000020504010101020606017f0141050b0722040366696200000673776974636800010462756c6b00020864697370"
    "6174636800040907010041000b01030a8f01051c002000420253047e200005200042017d1000200042027d10007c0b0b"
    "2200024002400240024020000e03000102030b410a0f0b41140f0b411e0f0b41e3000b390041e40041004105fc080000"
    "41c80141e4004105fc0a000041ac0241c1004103fc0b0041c80128000041ac022d00006a23006a410140006a0b070020"
    "0020016a0b0b002000200120021103000b0b1102010568656c6c6f0041100b0401020304";

static std::string unhex(const char* h) {
  std::string out;
  for (size_t i = 0; h[i] && h[i + 1]; i += 2) out.push_back((char)std::stoi(std::string(h + i, 2), nullptr, 16));
  return out;
}

static void test_wasm() {
  const std::string mod = unhex(kModuleHex);
  auto none = [](const std::string&, const std::string&, const wasm::FuncType&) { return wasm::HostFn{}; };
  {
    wasm::Instance in(wasm::Module::parse(mod), none);
    CHECK(in.invoke("fib", {20})[0] == 6765, "wasm: fib(20)");
    CHECK(in.invoke("switch", {1})[0] == 20 && in.invoke("switch", {7})[0] == 99, "wasm: br_table");
    const uint32_t want = (uint32_t)(0x6c6c6568u + 0x41u + 5u + 1u);
    CHECK((uint32_t)in.invoke("bulk", {})[0] == want, "wasm: bulk memory");
    CHECK(in.invoke("dispatch", {2, 3, 0})[0] == 5, "wasm: call_indirect");
    bool trapped = false;
    try {
      in.invoke("dispatch", {2, 3, 1});
    } catch (const wasm::Trap&) {
      trapped = true;
    }
    CHECK(trapped, "wasm: null table entry must trap");
  }
  std::mt19937 rng(11);
  int ran = 0, rejected = 0, trapped = 0, other = 0;
  for (int it = 0; it < 3000; ++it) {
    std::string m = mod;
    for (int k = 0, n = 1 + (int)(rng() % 3); k < n; ++k) m[rng() % m.size()] = (char)(rng() & 0xff);
    try {
      wasm::RunLimits lim;
      lim.fuel = 200000;
      lim.max_pages = 64;
      wasm::Instance in(wasm::Module::parse(m), none, lim);
      for (const char* f : {"fib", "switch", "bulk", "dispatch"}) {
        try {
          const uint32_t fi = in.export_func(f);
          std::vector<uint64_t> args(in.type_of(fi).params.size(), 3);
          in.call(fi, args);
          ++ran;
        } catch (const wasm::Trap&) {
          ++trapped;
        } catch (const wasm::LoadError&) {
          ++rejected;
        }
      }
    } catch (const wasm::LoadError&) {
      ++rejected;
    } catch (const wasm::Trap&) {
      ++trapped;
    } catch (const std::out_of_range& e) {
      ++other;
      if (getenv("SELFTEST_VERBOSE")) std::printf("out_of_range: %s\n", e.what());
    }
  }
  CHECK(ran > 0 && rejected > 0, "wasm fuzz: ran %d, rejected %d, trapped %d", ran, rejected, trapped);
  if (getenv("SELFTEST_VERBOSE")) std::printf("wasm fuzz: ran %d, rejected %d, trapped %d, other %d\n", ran, rejected, trapped, other);
}

// Suffix arrays against a plain sort, repeated substrings against their
// definition, and the Unigram lattice on random inputs (out-of-bounds reads
// show up under the address sanitizer).
static void test_text_index() {
  uint64_t seed = 0x9E3779B97F4A7C15ull;
  auto rnd = [&]() {
    seed ^= seed << 13;
    seed ^= seed >> 7;
    seed ^= seed << 17;
    return seed;
  };
  for (int trial = 0; trial < 300; ++trial) {
    const int n = (int)(rnd() % 200), k = 1 + (int)(rnd() % 5);
    std::vector<int32_t> s(n);
    for (auto& c : s) c = (int32_t)(rnd() % k) * 1000003;  // sparse symbol values
    const std::vector<int32_t> sa = text::suffix_array(s);
    std::vector<int32_t> ref(n);
    for (int i = 0; i < n; ++i) ref[i] = i;
    std::sort(ref.begin(), ref.end(), [&](int a, int b) {
      return std::lexicographical_compare(s.begin() + a, s.end(), s.begin() + b, s.end());
    });
    CHECK(sa == ref, "suffix array differs from a plain sort (n=%d)", n);
    const auto nodes = text::repeated_substrings(s);
    for (const auto& nd : nodes) {
      int count = 0;
      for (int i = 0; i + nd.length <= n; ++i)
        count += std::equal(s.begin() + nd.offset, s.begin() + nd.offset + nd.length, s.begin() + i);
      CHECK(count == nd.freq || nd.length == 0, "substring count %d != %d", count, nd.freq);
    }
    std::vector<std::u32string> pieces{U"a", U"b", U"c"};
    std::vector<double> scores{-1.0, -2.0, -3.0};
    for (int p = 0; p < 10; ++p) {
      std::u32string t;
      for (int j = 0, len = 2 + (int)(rnd() % 4); j < len; ++j) t.push_back(U'a' + (char32_t)(rnd() % 4));
      pieces.push_back(t);
      scores.push_back(-(double)(rnd() % 100) / 10.0);
    }
    pieces.push_back(U"<unk>");
    scores.push_back(0.0);
    text::UnigramModel m(pieces, scores, (int)pieces.size() - 1);
    std::u32string w;
    for (int j = 0, len = (int)(rnd() % 30); j < len; ++j) w.push_back(U'a' + (char32_t)(rnd() % 4));
    const auto ids = m.encode(w);
    size_t covered = 0;
    for (int32_t id : ids) covered += id == (int32_t)pieces.size() - 1 ? 1 : pieces[id].size();
    CHECK(covered == w.size(), "segmentation covers %zu of %zu", covered, w.size());
    std::vector<double> counts;
    m.expected_counts({w, w + U"ab"}, {1.0, 2.0}, counts);
    (void)m.alternative_scores();
  }
}

// HNSW: a batch insert linked by 4 threads (per-node locks), then one writer
// inserting while readers search (the index's lock); the nearest neighbour of
// an inserted vector is itself.
static void test_hnsw() {
  rag::Hnsw h(16, 8, 64, 3);
  std::mt19937 gen(5);
  std::normal_distribution<float> nd;
  std::vector<float> data(2000 * 16);
  for (auto& v : data) v = nd(gen);
  CHECK(h.add_batch(data.data(), 1000, 4) == 0, "hnsw: first label of a batch");  // 4 linking threads
  std::atomic<bool> done{false};
  std::vector<std::thread> readers;
  for (int t = 0; t < 3; ++t)
    readers.emplace_back([&, t] {
      std::vector<uint8_t> allow(2000, 1);
      while (!done.load())
        for (int i = 0; i < 50; ++i) (void)h.search(data.data() + 16 * ((i * 37 + t) % 2000), 5, 32, allow.data(), 2000);
    });
  for (int i = 1000; i < 2000; ++i) h.add(data.data() + 16 * i);
  done = true;
  for (auto& t : readers) t.join();
  int self = 0;
  for (int i = 0; i < 2000; i += 20) {
    auto r = h.search(data.data() + 16 * i, 1, 64, nullptr, 0);
    self += !r.empty() && r[0].second == i;
  }
  CHECK(self >= 95, "hnsw: only %d of 100 vectors find themselves", self);
  // saved graphs: random byte flips and truncations must make load() throw or
  // give a graph that searches without touching memory out of range
  const std::string path = "/tmp/kapsl-selftest-hnsw-" + std::to_string(getpid());
  h.save(path);
  std::string bytes;
  {
    std::FILE* f = std::fopen(path.c_str(), "rb");
    char buf[4096];
    for (size_t r; (r = std::fread(buf, 1, sizeof buf, f)) > 0;) bytes.append(buf, r);
    std::fclose(f);
  }
  CHECK(rag::Hnsw::load(path).size() == 2000, "hnsw: reloaded graph size");
  for (int trial = 0; trial < 40; ++trial) {
    std::string b = bytes;
    for (int k = 0; k < 4; ++k) b[gen() % b.size()] ^= (char)(1 + gen() % 255);
    if (trial % 5 == 0) b.resize(gen() % b.size());
    std::FILE* f = std::fopen(path.c_str(), "wb");
    std::fwrite(b.data(), 1, b.size(), f);
    std::fclose(f);
    try {
      rag::Hnsw g = rag::Hnsw::load(path);
      (void)g.search(data.data(), 5, 32, nullptr, 0);
    } catch (const std::exception&) {
    }
  }
  std::remove(path.c_str());
}

// A producer feeds 64 token channels in batches (append quietly, one post to the
// notifier thread per batch, like the engine loop); 64 consumers pop with bounded
// waits.  Every token arrives once and in order, and every stream ends.
static void test_token_channels() {
  constexpr int kChans = 64, kToks = 300;
  std::vector<std::shared_ptr<TokenChannel>> chans;
  for (int i = 0; i < kChans; ++i) chans.push_back(std::make_shared<TokenChannel>());
  std::vector<std::vector<int32_t>> got(kChans);
  std::vector<int> ends(kChans, 0);
  std::vector<std::thread> cons;
  for (int c = 0; c < kChans; ++c)
    cons.emplace_back([&, c] {
      std::vector<int32_t> out;
      std::string err;
      for (int spins = 0; spins < 20000; ++spins) {
        out.clear();
        const int r = chans[c]->pop(out, err, 50);
        got[c].insert(got[c].end(), out.begin(), out.end());
        if (r == TokenChannel::kEnd) {
          ends[c] = 1;
          return;
        }
      }
    });
  for (int t = 0; t < kToks; ++t) {
    std::vector<std::shared_ptr<TokenChannel>> batch;
    for (int c = 0; c < kChans; ++c) {
      chans[c]->push_quiet(c * 1000 + t, t == kToks - 1);
      batch.push_back(chans[c]);
    }
    TokenNotifier::get().post(std::move(batch));
  }
  for (auto& th : cons) th.join();
  for (int c = 0; c < kChans; ++c) {
    CHECK(ends[c] == 1, "channel %d did not end", c);
    bool ok = (int)got[c].size() == kToks;
    for (int t = 0; ok && t < kToks; ++t) ok = got[c][t] == c * 1000 + t;
    CHECK(ok, "channel %d: %zu tokens, wrong order or count", c, got[c].size());
  }
}

int main(int argc, char** argv) {
  const std::pair<const char*, void (*)()> tests[] = {
      {"ring_mpmc", test_ring_mpmc},         {"ring_repush", test_ring_repush}, {"model_pools", test_model_pools},
      {"shared_leases", test_shared_leases}, {"block_allocator", test_block_allocator}, {"wire", test_wire},
      {"cpu_pool", test_cpu_pool},           {"wasm", test_wasm},               {"text_index", test_text_index}, {"hnsw", test_hnsw},
      {"token_channels", test_token_channels}};
  for (auto& [name, fn] : tests) {
    if (argc > 1 && std::string(argv[1]) != name) continue;
    const auto t0 = std::chrono::steady_clock::now();
    fn();
    std::printf("%s %.2fs\n", name, std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count());
    std::fflush(stdout);
  }
  if (g_failures) {
    std::fprintf(stderr, "%d check(s) failed\n", g_failures);
    return 1;
  }
  std::printf("selftest ok\n");
  return 0;
}

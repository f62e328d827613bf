#include "text_index.h"

#include <algorithm>
#include <cmath>
#include <limits>
#include <stdexcept>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace kapsl {
namespace text {

namespace {

// Bucket boundaries of every symbol: its first slot (end=false) or one past
// its last slot (end=true).
void buckets(const int32_t* s, int32_t n, int32_t k, std::vector<int32_t>& b, bool end) {
  std::fill(b.begin(), b.end(), 0);
  for (int32_t i = 0; i < n; ++i) ++b[s[i]];
  int32_t sum = 0;
  for (int32_t c = 0; c < k; ++c) {
    sum += b[c];
    b[c] = end ? sum : sum - b[c];
  }
}

// Sorts the suffixes of s[0..n), where s[n-1] == 0 is the only 0 (the
// sentinel) and every symbol is below k.  sa has n slots; the reduced problem
// of the recursion reuses sa's upper part for its string.
void sais(const int32_t* s, int32_t* sa, int32_t n, int32_t k) {
  if (n == 1) {
    sa[0] = 0;
    return;
  }
  std::vector<uint8_t> stype(n);  // 1 = S-type suffix (smaller than the next one)
  stype[n - 1] = 1;
  for (int32_t i = n - 2; i >= 0; --i) stype[i] = s[i] < s[i + 1] || (s[i] == s[i + 1] && stype[i + 1]);
  auto lms = [&](int32_t i) { return i > 0 && stype[i] && !stype[i - 1]; };
  std::vector<int32_t> b(k);

  auto induce = [&]() {
    buckets(s, n, k, b, false);  // L-type suffixes, left to right, at bucket fronts
    for (int32_t i = 0; i < n; ++i) {
      const int32_t j = sa[i] - 1;
      if (sa[i] > 0 && !stype[j]) sa[b[s[j]]++] = j;
    }
    buckets(s, n, k, b, true);  // S-type suffixes, right to left, at bucket ends
    for (int32_t i = n - 1; i >= 0; --i) {
      const int32_t j = sa[i] - 1;
      if (sa[i] > 0 && stype[j]) sa[--b[s[j]]] = j;
    }
  };

  // 1. sort the LMS substrings: seed their positions at the bucket ends and induce
  buckets(s, n, k, b, true);
  std::fill(sa, sa + n, -1);
  for (int32_t i = 1; i < n; ++i)
    if (lms(i)) sa[--b[s[i]]] = i;
  induce();

  // 2. name them (equal substrings share a name), in the order of step 1
  int32_t n1 = 0;
  for (int32_t i = 0; i < n; ++i)
    if (lms(sa[i])) sa[n1++] = sa[i];
  std::fill(sa + n1, sa + n, -1);
  int32_t names = 0, prev = -1;
  for (int32_t i = 0; i < n1; ++i) {
    const int32_t pos = sa[i];
    bool differs = prev < 0;
    for (int32_t d = 0; !differs; ++d) {
      if (s[pos + d] != s[prev + d] || stype[pos + d] != stype[prev + d]) {
        differs = true;
      } else if (d > 0 && (lms(pos + d) || lms(prev + d))) {
        break;  // both substrings end here, equal
      }
    }
    if (differs) {
      ++names;
      prev = pos;
    }
    sa[n1 + pos / 2] = names - 1;  // LMS positions are at least 2 apart
  }
  for (int32_t i = n - 1, j = n - 1; i >= n1; --i)
    if (sa[i] >= 0) sa[j--] = sa[i];

  // 3. order of the LMS suffixes: recurse when names repeat
  int32_t* s1 = sa + n - n1;
  if (names < n1) {
    sais(s1, sa, n1, names);
  } else {
    for (int32_t i = 0; i < n1; ++i) sa[s1[i]] = i;
  }

  // 4. place the sorted LMS suffixes at their bucket ends and induce the rest
  for (int32_t i = 1, j = 0; i < n; ++i)
    if (lms(i)) s1[j++] = i;
  for (int32_t i = 0; i < n1; ++i) sa[i] = s1[sa[i]];
  std::fill(sa + n1, sa + n, -1);
  buckets(s, n, k, b, true);
  for (int32_t i = n1 - 1; i >= 0; --i) {
    const int32_t j = sa[i];
    sa[i] = -1;
    sa[--b[s[j]]] = j;
  }
  induce();
}

double log_add(double a, double b) {
  if (a == -INFINITY) return b;
  if (b == -INFINITY) return a;
  return a > b ? a + std::log1p(std::exp(b - a)) : b + std::log1p(std::exp(a - b));
}

}  // namespace

std::vector<int32_t> suffix_array(const std::vector<int32_t>& s) {
  const int32_t n = (int32_t)s.size();
  if (s.size() >= (size_t)std::numeric_limits<int32_t>::max() - 1) throw std::length_error("text too long");
  // rank the symbols densely (1..k-1) and append the sentinel 0
  std::vector<int32_t> alphabet(s);
  std::sort(alphabet.begin(), alphabet.end());
  alphabet.erase(std::unique(alphabet.begin(), alphabet.end()), alphabet.end());
  std::vector<int32_t> t(n + 1);
  for (int32_t i = 0; i < n; ++i)
    t[i] = 1 + (int32_t)(std::lower_bound(alphabet.begin(), alphabet.end(), s[i]) - alphabet.begin());
  t[n] = 0;
  std::vector<int32_t> sa(n + 1);
  sais(t.data(), sa.data(), n + 1, (int32_t)alphabet.size() + 1);
  return std::vector<int32_t>(sa.begin() + 1, sa.end());  // sa[0] is the sentinel
}

std::vector<int32_t> lcp_array(const std::vector<int32_t>& s, const std::vector<int32_t>& sa) {
  const int32_t n = (int32_t)s.size();
  std::vector<int32_t> rank(n), lcp(n, 0);
  for (int32_t i = 0; i < n; ++i) rank[sa[i]] = i;
  int32_t h = 0;
  for (int32_t i = 0; i < n; ++i) {
    if (rank[i] == 0) {
      h = 0;
      continue;
    }
    const int32_t j = sa[rank[i] - 1];
    while (i + h < n && j + h < n && s[i + h] == s[j + h]) ++h;
    lcp[rank[i]] = h;
    if (h > 0) --h;
  }
  return lcp;
}

std::vector<SubstringNode> repeated_substrings(const std::vector<int32_t>& s) {
  const int32_t n = (int32_t)s.size();
  std::vector<SubstringNode> out;
  if (n == 0) return out;
  const std::vector<int32_t> sa = suffix_array(s);
  const std::vector<int32_t> lcp = lcp_array(s, sa);
  std::vector<std::pair<int32_t, int32_t>> stack{{0, 0}};  // (lcp value, left bound)
  for (int32_t i = 1; i <= n; ++i) {
    const int32_t cur = i < n ? lcp[i] : -1;  // -1 flushes the root at the end
    int32_t lb = i - 1;
    while (!stack.empty() && cur < stack.back().first) {
      const auto [h, l] = stack.back();
      stack.pop_back();
      out.push_back({sa[l], h, i - l});
      lb = l;
    }
    if (cur >= 0 && (stack.empty() || cur > stack.back().first)) stack.push_back({cur, lb});
  }
  return out;
}

std::vector<SubstringNode> top_repeated_substrings(const std::vector<int32_t>& s, int32_t max_len, size_t limit,
                                                   const std::vector<int32_t>& banned,
                                                   const std::vector<int32_t>& not_inner) {
  const std::vector<SubstringNode> nodes = repeated_substrings(s);
  auto in = [](const std::vector<int32_t>& v, int32_t c) { return std::find(v.begin(), v.end(), c) != v.end(); };
  std::vector<std::pair<int64_t, int32_t>> keyed;  // (-freq * len, node index)
  for (size_t i = 0; i < nodes.size(); ++i) {
    const SubstringNode& nd = nodes[i];
    if (nd.length < 2 || nd.length > max_len) continue;
    bool ok = true;
    for (int32_t k = 0; k < nd.length && ok; ++k) {
      const int32_t c = s[nd.offset + k];
      ok = !in(banned, c) && (k == 0 || !in(not_inner, c));
    }
    if (ok) keyed.push_back({-(int64_t)nd.freq * nd.length, (int32_t)i});
  }
  const size_t k = std::min(limit, keyed.size());
  std::partial_sort(keyed.begin(), keyed.begin() + k, keyed.end());
  std::vector<SubstringNode> out;
  out.reserve(k);
  for (size_t i = 0; i < k; ++i) out.push_back(nodes[keyed[i].second]);
  return out;
}

// ------------------------------------------------------------------ Unigram
UnigramModel::UnigramModel(const std::vector<std::u32string>& pieces, const std::vector<double>& scores,
                           int unk_id)
    : pieces_(pieces), scores_(scores), unk_id_(unk_id) {
  if (pieces.size() != scores.size()) throw std::invalid_argument("pieces and scores differ in length");
  if (unk_id >= (int)pieces.size()) throw std::invalid_argument("unk_id out of range");
  double lo = 0.0;
  for (double v : scores) lo = std::min(lo, v);
  unk_score_ = lo - 10.0;
  trie_.emplace_back();
  // insert in lexicographic order: a node's children then arrive in code-point
  // order, so an existing child for c can only be the last one
  std::vector<int32_t> order(pieces.size());
  for (size_t p = 0; p < pieces.size(); ++p) order[p] = (int32_t)p;
  std::stable_sort(order.begin(), order.end(), [&](int32_t a, int32_t b) { return pieces[a] < pieces[b]; });
  for (int32_t p : order) {
    if (p == unk_id || pieces[p].empty()) continue;
    int32_t node = 0;
    for (char32_t c : pieces[p]) {
      auto& kids = trie_[node].kids;
      int32_t nxt = !kids.empty() && kids.back().first == c ? kids.back().second : -1;
      if (nxt < 0) {
        nxt = (int32_t)trie_.size();
        trie_[node].kids.push_back({c, nxt});
        trie_.emplace_back();
      }
      node = nxt;
    }
    if (trie_[node].piece < 0 || p < trie_[node].piece) trie_[node].piece = p;  // the lowest id of duplicates
  }
}

int32_t UnigramModel::child(int32_t node, char32_t c) const {
  const auto& k = trie_[node].kids;
  auto it = std::lower_bound(k.begin(), k.end(), std::make_pair(c, (int32_t)-1));
  return it != k.end() && it->first == c ? it->second : -1;
}

template <class F>
void UnigramModel::matches(const std::u32string& t, size_t i, F&& f) const {
  int32_t node = 0;
  bool single = false;
  for (size_t j = i; j < t.size(); ++j) {
    node = child(node, t[j]);
    if (node < 0) break;
    if (trie_[node].piece >= 0) {
      f(j + 1, trie_[node].piece, scores_[trie_[node].piece]);
      single |= j == i;
    }
  }
  if (!single && unk_id_ >= 0) f(i + 1, unk_id_, unk_score_);
}

std::vector<int32_t> UnigramModel::viterbi(const std::u32string& t, int32_t exclude) const {
  const size_t n = t.size();
  std::vector<double> best(n + 1, -INFINITY);
  std::vector<int32_t> from(n + 1, -1), piece(n + 1, -1);
  best[0] = 0.0;
  for (size_t i = 0; i < n; ++i) {
    if (best[i] == -INFINITY) continue;
    matches(t, i, [&](size_t j, int32_t p, double sc) {
      if (p == exclude) return;
      const double v = best[i] + sc;
      if (v > best[j]) {
        best[j] = v;
        from[j] = (int32_t)i;
        piece[j] = p;
      }
    });
  }
  if (best[n] == -INFINITY) return {};
  std::vector<int32_t> out;
  for (int32_t j = (int32_t)n; j > 0; j = from[j]) out.push_back(piece[j]);
  std::reverse(out.begin(), out.end());
  return out;
}

std::vector<int32_t> UnigramModel::encode(const std::u32string& text) const {
  if (text.empty()) return {};
  std::vector<int32_t> out = viterbi(text, -1);
  if (out.empty()) throw std::invalid_argument("text has characters that no piece covers and there is no unk piece");
  return out;
}

std::vector<int32_t> UnigramModel::alternative(int32_t p) const {
  if (p < 0 || p >= (int32_t)pieces_.size() || pieces_[p].size() <= 1) return {};
  return viterbi(pieces_[p], p);
}

std::vector<double> UnigramModel::alternative_scores() const {
  const int64_t n = (int64_t)pieces_.size();
  std::vector<double> out(n, -INFINITY);
#pragma omp parallel for schedule(dynamic, 256)
  for (int64_t p = 0; p < n; ++p) {
    if (pieces_[p].size() <= 1 || (int)p == unk_id_) continue;
    const std::vector<int32_t> alt = viterbi(pieces_[p], (int32_t)p);
    if (alt.empty()) continue;
    double v = 0.0;
    for (int32_t a : alt) v += a == unk_id_ ? unk_score_ : scores_[a];
    out[p] = v;
  }
  return out;
}

double UnigramModel::expected_counts(const std::vector<std::u32string>& words, const std::vector<double>& freqs,
                                     std::vector<double>& counts) const {
  if (words.size() != freqs.size()) throw std::invalid_argument("words and freqs differ in length");
  counts.assign(scores_.size(), 0.0);
  double loglik = 0.0;
  const int64_t W = (int64_t)words.size();
#pragma omp parallel
  {
    std::vector<double> local(scores_.size(), 0.0);
    std::vector<double> alpha, beta;
    struct Edge {
      int32_t i, j, p;
      double sc;
    };
    std::vector<Edge> edges;
    double ll = 0.0;
#pragma omp for schedule(dynamic, 64) nowait
    for (int64_t w = 0; w < W; ++w) {
      const std::u32string& t = words[w];
      const size_t n = t.size();
      if (n == 0) continue;
      alpha.assign(n + 1, -INFINITY);
      beta.assign(n + 1, -INFINITY);
      edges.clear();
      alpha[0] = 0.0;
      for (size_t i = 0; i < n; ++i) {
        if (alpha[i] == -INFINITY) continue;
        matches(t, i, [&](size_t j, int32_t p, double sc) {
          edges.push_back({(int32_t)i, (int32_t)j, p, sc});
          alpha[j] = log_add(alpha[j], alpha[i] + sc);
        });
      }
      const double z = alpha[n];
      if (z == -INFINITY) continue;  // no segmentation (no unk piece)
      beta[n] = 0.0;
      for (size_t e = edges.size(); e-- > 0;) beta[edges[e].i] = log_add(beta[edges[e].i], edges[e].sc + beta[edges[e].j]);
      for (const Edge& e : edges) {
        const double lp = alpha[e.i] + e.sc + beta[e.j] - z;
        if (lp > -700.0) local[e.p] += freqs[w] * std::exp(lp);
      }
      ll += freqs[w] * z;
    }
#pragma omp critical
    {
      for (size_t p = 0; p < local.size(); ++p) counts[p] += local[p];
      loglik += ll;
    }
  }
  return loglik;
}

}  // namespace text
}  // namespace kapsl

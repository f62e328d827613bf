// Text indexing for tokenizer training and Unigram tokenization.
//
// * suffix_array: SA-IS induced sorting (Nong, Zhang and Chan, "Two Efficient
//   Algorithms for Linear Time Suffix Array Construction", 2009) over any int32
//   alphabet (symbols are first ranked densely).
// * lcp_array: Kasai et al. 2001 (lcp[i] = common prefix of the suffixes at
//   sa[i-1] and sa[i]; lcp[0] = 0).
// * repeated_substrings: the lcp-intervals of the enhanced suffix array
//   (Abouelhoda, Kurtz and Ohlebusch 2004), i.e. the internal nodes of the
//   suffix tree, in bottom-up order with the root (the empty string, which
//   occurs n times) last.  Each is (offset of one occurrence, length, number
//   of occurrences).  This is what the reference's patched esaxx-rs returns
//   from `suffix()` (patches/esaxx-rs/src/lib.rs:110-215, esaxx.cpp:623).
// * UnigramModel: Viterbi segmentation and forward-backward expected piece
//   counts over a code-point trie of the pieces (Kudo, "Subword
//   Regularization", 2018), the two kernels of Unigram training.
#pragma once

#include <stdint.h>

#include <string>
#include <vector>

namespace kapsl {
namespace text {

std::vector<int32_t> suffix_array(const std::vector<int32_t>& s);
std::vector<int32_t> lcp_array(const std::vector<int32_t>& s, const std::vector<int32_t>& sa);

struct SubstringNode {
  int32_t offset, length, freq;
};
std::vector<SubstringNode> repeated_substrings(const std::vector<int32_t>& s);
// The `limit` repeated substrings of 2..max_len symbols with the largest
// freq * length (ties: earlier in bottom-up order first) that contain no
// symbol of `banned` and no symbol of `not_inner` after their first position.
std::vector<SubstringNode> top_repeated_substrings(const std::vector<int32_t>& s, int32_t max_len, size_t limit,
                                                   const std::vector<int32_t>& banned,
                                                   const std::vector<int32_t>& not_inner);

class UnigramModel {
 public:
  // unk_id: the piece emitted for a character that no piece covers (scored
  // min(scores) - 10); -1 makes such text an error.
  UnigramModel(const std::vector<std::u32string>& pieces, const std::vector<double>& scores, int unk_id);
  // Highest-scoring segmentation; ties keep the earlier-found (longer-prefix
  // first) path.
  std::vector<int32_t> encode(const std::u32string& text) const;
  // Adds freq * E[count of piece p in a segmentation of word] to counts[p]
  // for every word (lattice forward-backward in log space) and returns
  // sum(freq * log Z(word)).  Words are processed in parallel.
  double expected_counts(const std::vector<std::u32string>& words, const std::vector<double>& freqs,
                         std::vector<double>& counts) const;
  // Best segmentation of pieces[p] that does not use p itself (the
  // alternative whose likelihood replaces p's when p is pruned); empty when
  // the piece is a single character.
  std::vector<int32_t> alternative(int32_t p) const;
  // Score of alternative(p) for every piece (-inf for single characters and
  // pieces with no other segmentation); pieces are processed in parallel.
  std::vector<double> alternative_scores() const;
  size_t size() const { return scores_.size(); }

 private:
  struct Node {
    std::vector<std::pair<char32_t, int32_t>> kids;  // sorted by code point
    int32_t piece = -1;
  };
  int32_t child(int32_t node, char32_t c) const;
  template <class F>
  void matches(const std::u32string& t, size_t i, F&& f) const;  // f(end, piece) for every piece at t[i..]
  std::vector<int32_t> viterbi(const std::u32string& t, int32_t exclude) const;

  std::vector<Node> trie_;
  std::vector<std::u32string> pieces_;
  std::vector<double> scores_;
  int unk_id_;
  double unk_score_;
};

}  // namespace text
}  // namespace kapsl

// pk_text.h -- prompt text on the host: the pre-tokenizer patterns, the
// byte-level BPE tokenizer read from GGUF metadata, and the chat template.
//
// Follows rust/pocketinfer/src/regexlite.rs (the backtracking matcher the
// reference splits text with), tokenizer.rs (Tokenizer::from_gguf, encode,
// decode_token, is_eog) and chat.rs (apply_minicpm5, apply_generic).
#pragma once
#include <stddef.h>
#include <stdint.h>

#include <memory>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

namespace pk {

class Gguf;

namespace text {

// Unicode properties the pattern classes test (Rust's char::is_alphabetic,
// char::is_numeric and char::is_whitespace).
bool is_alphabetic(char32_t c);
bool is_numeric(char32_t c);
bool is_white_space(char32_t c);

// UTF-8 <-> code points.  utf8_decode fails on malformed input.
bool utf8_decode(const char *s, size_t n, std::u32string *out);
void utf8_append(std::string &out, char32_t c);

// One UTF-8 sequence at p[0 .. n): its length (1..4) when well formed; 0 and
// *bad = the length of its longest well-formed-so-far part (at least 1) when
// malformed; -1 when it is a well-formed prefix cut off by the end of p.
int utf8_sequence(const uint8_t *p, size_t n, size_t *bad);
// model.rs:1355-1388 flush_utf8: appends the ready text of pending to out
// (U+FFFD for each malformed sequence) and returns how many bytes of
// pending were consumed (the rest is an incomplete trailing sequence).
size_t utf8_flush(const uint8_t *pending, size_t n, std::string &out);

// A compiled pre-tokenizer pattern (regexlite.rs:1-481).
class Pattern {
 public:
  explicit Pattern(const std::u32string &src);
  ~Pattern();
  Pattern(const Pattern &) = delete;
  Pattern &operator=(const Pattern &) = delete;
  // End of the first alternative that matches at pos (leftmost-first,
  // greedy with backtracking), or -1.
  long match_at(const std::u32string &t, size_t pos) const;
  // Non-overlapping matches left to right; the scan stops at the first
  // position whose match is empty.
  std::vector<std::pair<size_t, size_t>> find(const std::u32string &t) const;

  struct Node;

 private:
  std::vector<std::vector<Node>> *alts_;
};

// Matches and the text between them, in order (regexlite.rs:461-481).
std::vector<std::u32string> split(const Pattern &p, const std::u32string &t);

class Tokenizer {
 public:
  // Tokenizer::from_gguf; returns false with err set when the metadata lacks
  // a token list.
  bool load(const Gguf &g, std::string &err);
  std::vector<uint32_t> encode(const std::string &utf8, bool parse_special) const;
  std::string token_bytes(uint32_t id) const;  // decode_token
  bool is_eog(uint32_t id) const;
  bool is_special(uint32_t id) const;

  size_t n_vocab() const { return tokens_.size(); }
  long bos_id() const { return bos_; }
  const std::vector<uint32_t> &eos_ids() const { return eos_; }
  const std::string &pre() const { return pre_; }
  bool ignore_merges() const { return ignore_merges_; }

 private:
  struct PairHash {
    size_t operator()(const std::pair<std::string, std::string> &p) const;
  };
  void encode_plain(const std::string &utf8, std::vector<uint32_t> &out) const;
  void encode_word(const std::u32string &word, std::vector<uint32_t> &out) const;

  std::vector<std::string> tokens_;
  std::vector<int32_t> types_;
  std::unordered_map<std::string, uint32_t> token_to_id_;
  std::unordered_map<std::pair<std::string, std::string>, uint32_t, PairHash> merges_;
  char32_t byte_to_char_[256] = {};
  std::unordered_map<char32_t, uint8_t> char_to_byte_;
  uint32_t byte_to_id_[256] = {};
  std::vector<std::pair<std::string, uint32_t>> specials_;  // longest first
  std::vector<std::shared_ptr<Pattern>> patterns_;
  std::string pre_;
  bool ignore_merges_ = false;
  long bos_ = -1;
  std::vector<uint32_t> eos_;
};

struct Message {
  std::string role, content;
};

// chat.rs:16-18, 20-97, 99-109.
bool is_minicpm5(const std::string &pre, const std::string &name);
std::string apply_minicpm5(const std::vector<Message> &m, bool add_generation_prompt);
std::string apply_generic(const std::vector<Message> &m, bool add_generation_prompt);
inline const char *direct_suffix() { return "<think>\n\n</think>\n\n"; }
inline const char *thinking_on_suffix() { return "<think>\n"; }

}  // namespace text
}  // namespace pk

// pk_text.cpp -- pre-tokenizer patterns, byte-level BPE, chat template.
//
// Host code: tokenisation is a short, branchy pass over a prompt's bytes and
// stays on the CPU beside the engine.  Every rule below restates the
// reference's behaviour (file:line in rust/pocketinfer/src/), including the
// corners where it differs from a general regex engine; those are named
// where they occur.
#include "pk_text.h"

#include <algorithm>
#include <climits>
#include <queue>

#include "pk_gguf.h"

namespace pk {
namespace text {

// ---------------------------------------------------------------- Unicode
#include "pk_unicode_tables.inc"

template <size_t N>
static bool in_ranges(const uint32_t (&r)[N][2], char32_t c) {
  size_t lo = 0, hi = N;
  while (lo < hi) {  // first range whose end is >= c
    const size_t mid = (lo + hi) / 2;
    if (r[mid][1] < (uint32_t)c) lo = mid + 1;
    else hi = mid;
  }
  return lo < N && r[lo][0] <= (uint32_t)c;
}

bool is_alphabetic(char32_t c) { return in_ranges(kAlphabetic, c); }
bool is_numeric(char32_t c) { return in_ranges(kNumeric, c); }
bool is_white_space(char32_t c) { return in_ranges(kWhiteSpace, c); }

bool utf8_decode(const char *s, size_t n, std::u32string *out) {
  const uint8_t *b = reinterpret_cast<const uint8_t *>(s);
  out->clear();
  out->reserve(n);
  size_t i = 0;
  while (i < n) {
    const uint8_t c0 = b[i];
    int len;
    char32_t cp, min;
    if (c0 < 0x80) { len = 1; cp = c0; min = 0; }
    else if ((c0 & 0xE0) == 0xC0) { len = 2; cp = c0 & 0x1F; min = 0x80; }
    else if ((c0 & 0xF0) == 0xE0) { len = 3; cp = c0 & 0x0F; min = 0x800; }
    else if ((c0 & 0xF8) == 0xF0) { len = 4; cp = c0 & 0x07; min = 0x10000; }
    else return false;
    if (i + len > n) return false;
    for (int k = 1; k < len; k++) {
      if ((b[i + k] & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (b[i + k] & 0x3F);
    }
    if (cp < min || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
    out->push_back(cp);
    i += len;
  }
  return true;
}

void utf8_append(std::string &o, char32_t c) {
  if (c < 0x80) {
    o.push_back((char)c);
  } else if (c < 0x800) {
    o.push_back((char)(0xC0 | (c >> 6)));
    o.push_back((char)(0x80 | (c & 0x3F)));
  } else if (c < 0x10000) {
    o.push_back((char)(0xE0 | (c >> 12)));
    o.push_back((char)(0x80 | ((c >> 6) & 0x3F)));
    o.push_back((char)(0x80 | (c & 0x3F)));
  } else {
    o.push_back((char)(0xF0 | (c >> 18)));
    o.push_back((char)(0x80 | ((c >> 12) & 0x3F)));
    o.push_back((char)(0x80 | ((c >> 6) & 0x3F)));
    o.push_back((char)(0x80 | (c & 0x3F)));
  }
}

// Well-formed sequences (the Unicode standard's table of UTF-8 byte
// sequences): the second byte's range depends on the lead byte, the others
// are 80..BF.
int utf8_sequence(const uint8_t *p, size_t n, size_t *bad) {
  const uint8_t c0 = p[0];
  int len;
  uint8_t lo = 0x80, hi = 0xBF;  // range of the second byte
  if (c0 < 0x80) return 1;
  if (c0 >= 0xC2 && c0 <= 0xDF) len = 2;
  else if (c0 == 0xE0) { len = 3; lo = 0xA0; }
  else if ((c0 >= 0xE1 && c0 <= 0xEC) || c0 == 0xEE || c0 == 0xEF) len = 3;
  else if (c0 == 0xED) { len = 3; hi = 0x9F; }
  else if (c0 == 0xF0) { len = 4; lo = 0x90; }
  else if (c0 >= 0xF1 && c0 <= 0xF3) len = 4;
  else if (c0 == 0xF4) { len = 4; hi = 0x8F; }
  else {
    *bad = 1;  // 80..C1, F5..FF never start a sequence
    return 0;
  }
  for (int i = 1; i < len; i++) {
    if ((size_t)i >= n) return -1;
    const uint8_t c = p[i];
    const bool ok = i == 1 ? (c >= lo && c <= hi) : (c >= 0x80 && c <= 0xBF);
    if (!ok) {
      *bad = (size_t)i;
      return 0;
    }
  }
  return len;
}

size_t utf8_flush(const uint8_t *p, size_t n, std::string &out) {
  size_t i = 0;
  while (i < n) {
    size_t bad = 0;
    const int len = utf8_sequence(p + i, n - i, &bad);
    if (len > 0) {
      out.append(reinterpret_cast<const char *>(p + i), (size_t)len);
      i += (size_t)len;
    } else if (len == 0) {
      out += "\xEF\xBF\xBD";  // U+FFFD
      i += bad;
    } else {
      break;  // an incomplete sequence at the end waits for the next bytes
    }
  }
  return i;
}

static std::string to_utf8(const std::u32string &s) {
  std::string o;
  o.reserve(s.size());
  for (char32_t c : s) utf8_append(o, c);
  return o;
}

// ---------------------------------------------------------------- patterns
namespace {

constexpr size_t kNoMax = SIZE_MAX;

// Class members (regexlite.rs:1-10).  kNotCr is what "\S" means inside
// brackets there: any character but '\r'.
enum ItemKind : uint8_t { kCh, kRange, kLetter, kNumber, kSpace, kNotCr, kNotLf };
struct Item {
  ItemKind kind;
  char32_t a, b;
};

}  // namespace

struct Pattern::Node {
  enum Kind : uint8_t { Char, Class, Any, Group, Repeat, Look } kind = Char;
  char32_t ch = 0;
  bool neg = false;
  std::vector<Item> items;
  std::vector<std::vector<Node>> alts;  // Group, Look
  std::vector<Node> sub;                // Repeat: the repeated node
  size_t min = 0, max = kNoMax;
};

namespace {

using Node = Pattern::Node;

Node class_node(bool neg, std::vector<Item> items) {
  Node n;
  n.kind = Node::Class;
  n.neg = neg;
  n.items = std::move(items);
  return n;
}

Node char_node(char32_t c) {
  Node n;
  n.kind = Node::Char;
  n.ch = c;
  return n;
}

// Recursive-descent parser of the pattern syntax regexlite.rs:28-270 accepts.
struct Parser {
  const std::u32string &c;
  size_t o = 0;

  bool more() const { return o < c.size(); }
  char32_t peek() const { return c[o]; }
  bool peek_is(char32_t x) const { return o < c.size() && c[o] == x; }

  std::vector<std::vector<Node>> alts(bool in_group) {  // :43-63
    std::vector<std::vector<Node>> out;
    std::vector<Node> seq;
    while (more()) {
      if (in_group && peek() == U')') break;
      if (peek() == U'|') {
        o++;
        out.push_back(std::move(seq));
        seq.clear();
        continue;
      }
      Node n;
      if (atom(&n)) seq.push_back(std::move(n));
    }
    out.push_back(std::move(seq));
    return out;
  }

  void expect(char32_t x) {
    if (peek_is(x)) o++;
  }

  std::u32string brace_name() {  // the name of \p{...}; the '{' is consumed already
    std::u32string name;
    while (more()) {
      const char32_t x = c[o++];
      if (x == U'}') break;
      name.push_back(x);
    }
    return name;
  }

  static bool is_letter_name(const std::u32string &n) {
    return n == U"L" || n == U"Lu" || n == U"Ll" || n == U"Lt" || n == U"Lm" || n == U"Lo";
  }

  bool atom(Node *out) {  // :64-146; false when the pattern ends inside an escape
    const char32_t ch = c[o++];
    Node base;
    if (ch == U'(') {
      base.kind = Node::Group;
      if (peek_is(U'?')) {
        o++;
        if (peek_is(U':')) {
          o++;
        } else if (peek_is(U'!') || peek_is(U'=')) {
          base.kind = Node::Look;
          base.neg = peek() == U'!';
          o++;
        }  // any other "(?x": x stays and is part of the group
      }
      base.alts = alts(true);
      expect(U')');
    } else if (ch == U'[') {
      base = bracket();
    } else if (ch == U'.') {
      base.kind = Node::Any;
    } else if (ch == U'\\') {
      if (!more()) return false;
      const char32_t e = c[o++];
      switch (e) {
        case U'p':
          if (peek_is(U'{')) {
            o++;
            const std::u32string name = brace_name();
            if (is_letter_name(name)) base = class_node(false, {{kLetter, 0, 0}});
            else if (name == U"N") base = class_node(false, {{kNumber, 0, 0}});
            else base = class_node(false, {});  // \p{P}, \p{S}, \p{M}, others: matches nothing
          } else {
            base = char_node(U'p');
          }
          break;
        case U's': base = class_node(false, {{kSpace, 0, 0}}); break;
        case U'S': base = class_node(true, {{kSpace, 0, 0}}); break;
        case U'd': base = class_node(false, {{kRange, U'0', U'9'}}); break;
        case U'w':
          base = class_node(false, {{kRange, U'a', U'z'}, {kRange, U'A', U'Z'}, {kRange, U'0', U'9'}, {kCh, U'_', 0}});
          break;
        case U'r': base = char_node(U'\r'); break;
        case U'n': base = char_node(U'\n'); break;
        case U't': base = char_node(U'\t'); break;
        default: base = char_node(e); break;
      }
    } else {
      base = char_node(ch);
    }
    *out = quant(std::move(base));
    return true;
  }

  static size_t digits_value(const std::u32string &d, size_t overflow) {
    size_t v = 0;
    for (char32_t x : d) {
      if (v > (SIZE_MAX - 9) / 10) return overflow;
      v = v * 10 + (size_t)(x - U'0');
    }
    return v;
  }

  Node quant(Node base) {  // :147-209
    size_t mn, mx;
    if (peek_is(U'*')) { o++; mn = 0; mx = kNoMax; }
    else if (peek_is(U'+')) { o++; mn = 1; mx = kNoMax; }
    else if (peek_is(U'?')) { o++; mn = 0; mx = 1; }
    else if (peek_is(U'{')) {
      const size_t save = o;
      o++;
      std::u32string a, b;
      while (more() && peek() >= U'0' && peek() <= U'9') a.push_back(c[o++]);
      bool comma = false;
      if (peek_is(U',')) {
        comma = true;
        o++;
        while (more() && peek() >= U'0' && peek() <= U'9') b.push_back(c[o++]);
      }
      if (peek_is(U'}') && (!a.empty() || comma)) {
        o++;
        mn = digits_value(a, 0);  // an unparsable count reads as 0
        mx = b.empty() ? (comma ? kNoMax : mn) : digits_value(b, kNoMax);
      } else {
        o = save;
        return base;
      }
    } else {
      return base;
    }
    if (peek_is(U'?')) o++;  // a lazy marker is read and ignored: repeats stay greedy
    Node r;
    r.kind = Node::Repeat;
    r.min = mn;
    r.max = mx;
    r.sub.push_back(std::move(base));
    return r;
  }

  Node bracket() {  // :210-263
    const bool neg = peek_is(U'^');
    if (neg) o++;
    std::vector<Item> items;
    while (more()) {
      const char32_t x = c[o++];
      if (x == U']') break;
      if (x == U'\\') {
        const char32_t e = more() ? c[o++] : U'\\';
        switch (e) {
          case U's': items.push_back({kSpace, 0, 0}); break;
          case U'S': items.push_back({kNotCr, 0, 0}); break;
          case U'd': items.push_back({kRange, U'0', U'9'}); break;
          case U'r': items.push_back({kCh, U'\r', 0}); break;
          case U'n': items.push_back({kCh, U'\n', 0}); break;
          case U't': items.push_back({kCh, U'\t', 0}); break;
          case U'p':
            if (peek_is(U'{')) {
              o++;
              const std::u32string name = brace_name();
              if (is_letter_name(name)) items.push_back({kLetter, 0, 0});
              else if (name == U"N") items.push_back({kNumber, 0, 0});
            }
            break;
          default: items.push_back({kCh, e, 0}); break;
        }
        continue;
      }
      if (peek_is(U'-') && !(o + 1 < c.size() && c[o + 1] == U']')) {
        o++;
        char32_t hi = U'-';
        if (more()) {
          const char32_t h = c[o++];
          if (h == U'\\') {
            if (more()) {
              const char32_t e = c[o++];
              hi = e == U'r' ? U'\r' : e == U'n' ? U'\n' : e == U't' ? U'\t' : e;
            }
          } else {
            hi = h;
          }
        }
        items.push_back({kRange, x, hi});
      } else {
        items.push_back({kCh, x, 0});
      }
    }
    return class_node(neg, std::move(items));
  }
};

bool class_match(const Node &n, char32_t c) {  // :278-297
  bool hit = false;
  for (const Item &it : n.items) {
    bool m = false;
    switch (it.kind) {
      case kCh: m = c == it.a; break;
      case kRange: m = c >= it.a && c <= it.b; break;
      case kLetter: m = is_alphabetic(c); break;
      case kNumber: m = is_numeric(c); break;
      case kSpace: m = is_white_space(c); break;
      case kNotCr: m = c != U'\r'; break;
      case kNotLf: m = c != U'\n'; break;
    }
    if (m) {
      hit = true;
      break;
    }
  }
  return hit != n.neg;
}

// A borrowed "what to match next" callback: continuation-passing lets the
// matcher backtrack into repeats and alternatives exactly as :299-402 do.
struct Cont {
  const void *obj;
  bool (*fn)(const void *, size_t);
  bool operator()(size_t p) const { return fn(obj, p); }
};
template <class F>
Cont cont(const F &f) {
  return Cont{&f, [](const void *o, size_t p) { return (*static_cast<const F *>(o))(p); }};
}

struct Matcher {
  const std::u32string &t;

  bool seq(const Node *n, size_t cnt, size_t pos, Cont k) const {
    if (cnt == 0) return k(pos);
    const Node &nd = n[0];
    switch (nd.kind) {
      case Node::Char:
        return pos < t.size() && t[pos] == nd.ch && seq(n + 1, cnt - 1, pos + 1, k);
      case Node::Any:
        return pos < t.size() && t[pos] != U'\n' && t[pos] != U'\r' && seq(n + 1, cnt - 1, pos + 1, k);
      case Node::Class:
        return pos < t.size() && class_match(nd, t[pos]) && seq(n + 1, cnt - 1, pos + 1, k);
      case Node::Group: {
        const auto rest = [&](size_t p2) { return seq(n + 1, cnt - 1, p2, k); };
        for (const auto &alt : nd.alts)
          if (seq(alt.data(), alt.size(), pos, cont(rest))) return true;
        return false;
      }
      case Node::Look: {  // a lookahead: any alternative matching at pos, nothing consumed
        const auto any = [](size_t) { return true; };
        bool matched = false;
        for (const auto &alt : nd.alts)
          if (seq(alt.data(), alt.size(), pos, cont(any))) {
            matched = true;
            break;
          }
        if (matched == nd.neg) return false;
        return seq(n + 1, cnt - 1, pos, k);
      }
      case Node::Repeat:
        return rep(nd, n + 1, cnt - 1, pos, 0, k);
    }
    return false;
  }

  static bool one(const Node &nd, char32_t c) {
    return nd.kind == Node::Char ? c == nd.ch : nd.kind == Node::Any ? (c != U'\n' && c != U'\r') : class_match(nd, c);
  }

  // Greedy: one more of the node (it must consume something) before the
  // rest; a repeated repeat or lookahead never repeats (:354-395).
  bool rep(const Node &r, const Node *rest, size_t rc, size_t pos, size_t count, Cont k) const {
    const Node &node = r.sub[0];
    if (count == 0 && (node.kind == Node::Char || node.kind == Node::Any || node.kind == Node::Class)) {
      // A one-character node: the recursion below would take the longest run
      // and then try the rest after c = run, run - 1, ..., min characters.
      // The same order as a loop, so a long run of letters or spaces costs no
      // stack depth.
      const size_t lim = r.max == kNoMax ? t.size() - pos : std::min(r.max, t.size() - pos);
      size_t m = 0;
      while (m < lim && one(node, t[pos + m])) m++;
      for (size_t c = m + 1; c-- > 0;)
        if (c >= r.min && seq(rest, rc, pos + c, k)) return true;
      return false;
    }
    const bool can_more = r.max == kNoMax || count < r.max;
    if (can_more && node.kind != Node::Repeat && node.kind != Node::Look) {
      const auto next = [&](size_t p2) { return p2 != pos && rep(r, rest, rc, p2, count + 1, k); };
      if (seq(&node, 1, pos, cont(next))) return true;
    }
    return count >= r.min && seq(rest, rc, pos, k);
  }
};

}  // namespace

Pattern::Pattern(const std::u32string &src) {
  Parser p{src};
  alts_ = new std::vector<std::vector<Node>>(p.alts(false));
}

Pattern::~Pattern() { delete alts_; }

long Pattern::match_at(const std::u32string &t, size_t pos) const {  // :406-418
  Matcher m{t};
  for (const auto &alt : *alts_) {
    size_t end = 0;
    const auto rec = [&](size_t p) {
      end = p;
      return true;
    };
    if (m.seq(alt.data(), alt.size(), pos, cont(rec))) return (long)end;
  }
  return -1;
}

std::vector<std::pair<size_t, size_t>> Pattern::find(const std::u32string &t) const {  // :420-446
  std::vector<std::pair<size_t, size_t>> out;
  size_t i = 0;
  while (i < t.size()) {
    bool found = false;
    size_t s = 0, e = 0;
    for (size_t j = i; j < t.size(); j++) {
      const long end = match_at(t, j);
      if (end >= 0) {
        if ((size_t)end > j) {
          found = true;
          s = j;
          e = (size_t)end;
        }
        break;  // an empty match ends the whole scan
      }
    }
    if (!found) break;
    out.emplace_back(s, e);
    i = e;
  }
  return out;
}

std::vector<std::u32string> split(const Pattern &p, const std::u32string &t) {
  std::vector<std::u32string> out;
  size_t last = 0;
  for (const auto &m : p.find(t)) {
    if (m.first > last) out.push_back(t.substr(last, m.first - last));
    out.push_back(t.substr(m.first, m.second - m.first));
    last = m.second;
  }
  if (last < t.size()) out.push_back(t.substr(last));
  if (out.empty()) out.emplace_back();
  return out;
}

// ---------------------------------------------------------------- tokenizer
namespace {

// Pre-tokenizer patterns by tokenizer.ggml.pre (tokenizer.rs:6-22, 262-270).
const char32_t *const kPreMiniCpm5[] = {
    U"\\p{N}{1,3}",
    U"(?:'[sS]|'[tT]|'[rR][eE]|'[vV][eE]|'[mM]|'[lL][lL]|'[dD])|[^\\r\\n\\p{L}\\p{N}]?\\p{L}+|\\p{N}+| ?[^\\s\\p{L}"
    U"\\p{N}]+[\\r\\n]*|\\s*[\\r\\n]+|\\s+(?!\\S)|\\s+"};
const char32_t *const kPreQwen2[] = {
    U"(?:'[sS]|'[tT]|'[rR][eE]|'[vV][eE]|'[mM]|'[lL][lL]|'[dD])|[^\\r\\n\\p{L}\\p{N}]?\\p{L}+|\\p{N}+| ?[^\\s\\p{L}"
    U"\\p{N}]+[\\r\\n]*|\\s*[\\r\\n]+|\\s+(?!\\S)|\\s+"};
const char32_t *const kPreGpt2[] = {U"'s|'t|'re|'ve|'m|'ll|'d| ?\\p{L}+| ?\\p{N}+| ?[^\\s\\p{L}\\p{N}]+|\\s+(?!\\S)"};
const char32_t *const kPreLlama3[] = {
    U"(?:'[sS]|'[tT]|'[rR][eE]|'[vV][eE]|'[mM]|'[lL][lL]|'[dD])|[^\\r\\n\\p{L}\\p{N}]?\\p{L}+|\\p{N}{1,3}| ?[^\\s"
    U"\\p{L}\\p{N}]+[\\r\\n]*|\\s*[\\r\\n]+|\\s+(?!\\S)|\\s+"};

std::vector<std::shared_ptr<Pattern>> patterns_for(const std::string &pre) {
  std::vector<const char32_t *> src;
  if (pre == "minicpm5") src.assign(std::begin(kPreMiniCpm5), std::end(kPreMiniCpm5));
  else if (pre == "qwen2" || pre == "qwen2.5" || pre == "qwen3") src.assign(std::begin(kPreQwen2), std::end(kPreQwen2));
  else if (pre == "llama3" || pre == "llama-bpe" || pre == "llama-v3")
    src.assign(std::begin(kPreLlama3), std::end(kPreLlama3));
  else src.assign(std::begin(kPreGpt2), std::end(kPreGpt2));  // "gpt-2", "phi-2" and anything else
  std::vector<std::shared_ptr<Pattern>> out;
  for (const char32_t *s : src) out.push_back(std::make_shared<Pattern>(std::u32string(s)));
  return out;
}

bool is_special_type(int32_t t) { return t == 2 || t == 3 || t == 4; }

}  // namespace

size_t Tokenizer::PairHash::operator()(const std::pair<std::string, std::string> &p) const {
  const size_t a = std::hash<std::string>()(p.first), b = std::hash<std::string>()(p.second);
  return a ^ (b + 0x9E3779B97F4A7C15ull + (a << 6) + (a >> 2));
}

bool Tokenizer::load(const Gguf &g, std::string &err) {  // tokenizer.rs:38-110
  const GgufValue *tv = g.get("tokenizer.ggml.tokens");
  if (!tv || tv->type != 9 || tv->arr_type != 8) {
    err = "metadata tokenizer.ggml.tokens is not a string array";
    return false;
  }
  tokens_ = tv->arr_str;
  const size_t n = tokens_.size();
  const GgufValue *ty = g.get("tokenizer.ggml.token_type");
  if (ty && ty->type == 9 && ty->arr_type == 5) types_ = ty->arr_i32;
  else types_.assign(n, 1);  // no i32 type array: every token normal
  if (types_.size() < n) {
    err = "tokenizer.ggml.token_type has fewer entries than tokenizer.ggml.tokens";
    return false;
  }
  // merges: "left right", split at the first space after the first byte;
  // rank = index, a later duplicate pair taking the later rank
  merges_.clear();
  if (const GgufValue *mv = g.get("tokenizer.ggml.merges"))
    if (mv->type == 9 && mv->arr_type == 8)
      for (size_t i = 0; i < mv->arr_str.size(); i++) {
        const std::string &m = mv->arr_str[i];
        const size_t sp = m.size() > 1 ? m.find(' ', 1) : std::string::npos;
        if (sp == std::string::npos) continue;
        merges_[{m.substr(0, sp), m.substr(sp + 1)}] = (uint32_t)i;
      }
  // the byte <-> character map of byte-level BPE (:275-300): printable
  // Latin-1 bytes map to themselves, the other 68 bytes to U+0100.. in order
  bool direct[256] = {};
  for (int b = '!'; b <= '~'; b++) direct[b] = true;
  for (int b = 0xA1; b <= 0xAC; b++) direct[b] = true;
  for (int b = 0xAE; b <= 0xFF; b++) direct[b] = true;
  char_to_byte_.clear();
  char32_t extra = 256;
  for (int b = 0; b < 256; b++) {
    byte_to_char_[b] = direct[b] ? (char32_t)b : extra++;
    char_to_byte_[byte_to_char_[b]] = (uint8_t)b;
  }
  token_to_id_.clear();
  token_to_id_.reserve(n);
  std::fill(std::begin(byte_to_id_), std::end(byte_to_id_), UINT32_MAX);
  std::u32string cs;
  for (size_t i = 0; i < n; i++) {
    token_to_id_.emplace(tokens_[i], (uint32_t)i);  // the first id of a repeated token wins
    if (utf8_decode(tokens_[i].data(), tokens_[i].size(), &cs) && cs.size() == 1) {
      const auto it = char_to_byte_.find(cs[0]);
      if (it != char_to_byte_.end() && byte_to_id_[it->second] == UINT32_MAX) byte_to_id_[it->second] = (uint32_t)i;
    }
  }
  specials_.clear();
  for (size_t i = 0; i < n; i++)
    if (is_special_type(types_[i])) specials_.emplace_back(tokens_[i], (uint32_t)i);
  std::stable_sort(specials_.begin(), specials_.end(),
                   [](const auto &a, const auto &b) { return a.first.size() > b.first.size(); });
  pre_ = g.get_str("tokenizer.ggml.pre");
  patterns_ = patterns_for(pre_);
  ignore_merges_ = pre_ == "minicpm5";
  uint64_t v;
  bos_ = g.get_u64("tokenizer.ggml.bos_token_id", &v) ? (long)(uint32_t)v : -1;
  eos_.clear();
  if (g.get_u64("tokenizer.ggml.eos_token_id", &v)) eos_.push_back((uint32_t)v);
  for (const auto &s : specials_)
    if (s.first == "<|im_end|>" || s.first == "<|eot|>" || s.first == "<|endoftext|>") eos_.push_back(s.second);
  std::sort(eos_.begin(), eos_.end());
  eos_.erase(std::unique(eos_.begin(), eos_.end()), eos_.end());
  return true;
}

// One pre-tokenized word (tokenizer.rs:112-169): its UTF-8 bytes through the
// byte map; the whole word as one token when merges are ignored and it is a
// token; else pairwise merges, lowest rank first (leftmost on equal rank),
// then each symbol's id, or its characters' ids, or the byte tokens.
void Tokenizer::encode_word(const std::u32string &word, std::vector<uint32_t> &out) const {
  std::u32string mapped;
  std::string bytes = to_utf8(word);
  mapped.reserve(bytes.size());
  for (unsigned char b : bytes) mapped.push_back(byte_to_char_[b]);
  if (ignore_merges_) {
    const auto it = token_to_id_.find(to_utf8(mapped));
    if (it != token_to_id_.end()) {
      out.push_back(it->second);
      return;
    }
  }
  // Symbols as a linked list (indexed by their first character) and a heap
  // of candidate pairs ordered by (rank, position): popping the smallest
  // still-current pair is the reference's "lowest rank, leftmost" pick, in
  // O(n log n) instead of a rescan per merge.  A pair is stale once either
  // side has changed (version numbers).
  const size_t n = mapped.size();
  std::vector<std::string> sym(n);
  for (size_t i = 0; i < n; i++) utf8_append(sym[i], mapped[i]);
  std::vector<long> nxt(n), prv(n);
  std::vector<uint32_t> ver(n, 0);
  for (size_t i = 0; i < n; i++) {
    nxt[i] = i + 1 < n ? (long)(i + 1) : -1;
    prv[i] = (long)i - 1;
  }
  struct Cand {
    uint32_t rank;
    size_t left, right;
    uint32_t vl, vr;
  };
  const auto later = [](const Cand &a, const Cand &b) { return a.rank != b.rank ? a.rank > b.rank : a.left > b.left; };
  std::priority_queue<Cand, std::vector<Cand>, decltype(later)> heap(later);
  const auto push = [&](size_t l) {
    const long r = nxt[l];
    if (r < 0) return;
    const auto it = merges_.find({sym[l], sym[(size_t)r]});
    if (it != merges_.end()) heap.push(Cand{it->second, l, (size_t)r, ver[l], ver[(size_t)r]});
  };
  for (size_t i = 0; i + 1 < n; i++) push(i);
  while (!heap.empty()) {
    const Cand c = heap.top();
    heap.pop();
    if (ver[c.left] != c.vl || ver[c.right] != c.vr || nxt[c.left] != (long)c.right) continue;
    sym[c.left] += sym[c.right];
    sym[c.right].clear();
    ver[c.left]++;
    ver[c.right]++;
    nxt[c.left] = nxt[c.right];
    if (nxt[c.right] >= 0) prv[(size_t)nxt[c.right]] = (long)c.left;
    if (prv[c.left] >= 0) push((size_t)prv[c.left]);
    push(c.left);
  }
  std::vector<std::string> merged;
  for (long i = n ? 0 : -1; i >= 0; i = nxt[(size_t)i]) merged.push_back(std::move(sym[(size_t)i]));
  sym.swap(merged);
  std::u32string cs;
  for (const std::string &s : sym) {
    const auto it = token_to_id_.find(s);
    if (it != token_to_id_.end()) {
      out.push_back(it->second);
      continue;
    }
    utf8_decode(s.data(), s.size(), &cs);  // symbols are whole characters
    for (char32_t ch : cs) {
      std::string one;
      utf8_append(one, ch);
      const auto ic = token_to_id_.find(one);
      if (ic != token_to_id_.end()) {
        out.push_back(ic->second);
      } else {
        const auto ib = char_to_byte_.find(ch);
        if (ib != char_to_byte_.end() && byte_to_id_[ib->second] != UINT32_MAX) out.push_back(byte_to_id_[ib->second]);
      }
    }
  }
}

// tokenizer.rs:171-185: every pattern in turn splits every piece (matches and
// the text between them; empty pieces dropped), then each word is encoded.
void Tokenizer::encode_plain(const std::string &utf8, std::vector<uint32_t> &out) const {
  std::u32string all;
  utf8_decode(utf8.data(), utf8.size(), &all);
  std::vector<std::u32string> words{all};
  for (const auto &pat : patterns_) {
    std::vector<std::u32string> next;
    for (const auto &w : words)
      for (auto &part : split(*pat, w))
        if (!part.empty()) next.push_back(std::move(part));
    words.swap(next);
  }
  for (const auto &w : words) encode_word(w, out);
}

// tokenizer.rs:187-224: with parse_special, the longest special token text
// starting at each character boundary is emitted as its id and the text
// between specials is encoded plainly.
std::vector<uint32_t> Tokenizer::encode(const std::string &text, bool parse_special) const {
  std::vector<uint32_t> out;
  if (!parse_special || specials_.empty()) {
    encode_plain(text, out);
    return out;
  }
  size_t pos = 0, plain = 0;
  const size_t n = text.size();
  while (pos < n) {
    const std::pair<std::string, uint32_t> *hit = nullptr;
    for (const auto &s : specials_)
      if (!s.first.empty() && pos + s.first.size() <= n && text.compare(pos, s.first.size(), s.first) == 0) {
        hit = &s;
        break;
      }
    if (hit) {
      if (plain < pos) encode_plain(text.substr(plain, pos - plain), out);
      out.push_back(hit->second);
      pos += hit->first.size();
      plain = pos;
    } else {
      const unsigned char c0 = (unsigned char)text[pos];
      pos += c0 < 0x80 ? 1 : c0 < 0xE0 ? 2 : c0 < 0xF0 ? 3 : 4;
    }
  }
  if (plain < n) encode_plain(text.substr(plain), out);
  return out;
}

std::string Tokenizer::token_bytes(uint32_t id) const {  // tokenizer.rs:226-250
  if (id >= tokens_.size()) return std::string();
  const std::string &tok = tokens_[id];
  if (is_special_type(types_[id])) return tok;
  std::u32string cs;
  if (!utf8_decode(tok.data(), tok.size(), &cs)) return tok;
  std::string out;
  for (char32_t ch : cs) {
    const auto it = char_to_byte_.find(ch);
    if (it != char_to_byte_.end()) out.push_back((char)it->second);
    else utf8_append(out, ch);
  }
  return out;
}

bool Tokenizer::is_eog(uint32_t id) const { return std::binary_search(eos_.begin(), eos_.end(), id); }

bool Tokenizer::is_special(uint32_t id) const { return id < types_.size() && is_special_type(types_[id]); }

// ---------------------------------------------------------------- chat template
namespace {

bool contains(const std::string &s, const char *x) { return s.find(x) != std::string::npos; }

std::string before_first(const std::string &s, const std::string &sep) {
  const size_t p = s.find(sep);
  return p == std::string::npos ? s : s.substr(0, p);
}

// The piece after the last separator (the separators here cannot overlap
// themselves, so this equals the last piece of a left-to-right split).
std::string after_last(const std::string &s, const std::string &sep) {
  const size_t p = s.rfind(sep);
  return p == std::string::npos ? s : s.substr(p + sep.size());
}

std::string lstrip_nl(const std::string &s) {
  const size_t p = s.find_first_not_of('\n');
  return p == std::string::npos ? std::string() : s.substr(p);
}

std::string rstrip_nl(const std::string &s) {
  const size_t p = s.find_last_not_of('\n');
  return p == std::string::npos ? std::string() : s.substr(0, p + 1);
}

}  // namespace

bool is_minicpm5(const std::string &pre, const std::string &name) {
  if (pre == "minicpm5") return true;
  std::string low = name;
  for (char &c : low)
    if (c >= 'A' && c <= 'Z') c = (char)(c - 'A' + 'a');
  return low.find("minicpm5") != std::string::npos;
}

// chat.rs:20-83.  A leading system turn first; user turns (and later system
// turns) as <|im_start|>role; assistant turns with their reasoning moved into
// a <think> block (an empty one when there is none); a run of tool turns as
// one user turn of <tool_response> blocks; other roles dropped.
std::string apply_minicpm5(const std::vector<Message> &m, bool add_generation_prompt) {
  std::string out = "<s>";
  if (!m.empty() && m[0].role == "system") out += "<|im_start|>system\n" + m[0].content + "<|im_end|>\n";
  size_t i = 0;
  while (i < m.size()) {
    const Message &x = m[i];
    if (x.role == "user" || (x.role == "system" && i > 0)) {
      out += "<|im_start|>" + x.role + "\n" + x.content + "<|im_end|>\n";
    } else if (x.role == "assistant") {
      std::string content = x.content, reasoning;
      if (contains(content, "</think>")) {
        reasoning = rstrip_nl(after_last(before_first(content, "</think>"), "<think>"));
        content = lstrip_nl(after_last(content, "</think>"));
      }
      out += "<|im_start|>assistant\n";
      if (!reasoning.empty()) {
        out += "<think>\n" + rstrip_nl(lstrip_nl(reasoning)) + "\n</think>\n\n" + lstrip_nl(content);
      } else if (!contains(content, "<think>") && !contains(content, "</think>")) {
        out += "<think>\n\n</think>\n\n" + lstrip_nl(content);
      } else {
        out += content;
      }
      out += "<|im_end|>\n";
    } else if (x.role == "tool") {
      out += "<|im_start|>user";
      while (i < m.size() && m[i].role == "tool") {
        out += "\n<tool_response>\n" + m[i].content + "\n</tool_response>";
        i++;
      }
      out += "<|im_end|>\n";
      continue;
    }
    i++;
  }
  if (add_generation_prompt) out += "<|im_start|>assistant\n";
  return out;
}

std::string apply_generic(const std::vector<Message> &m, bool add_generation_prompt) {  // chat.rs:85-97
  std::string out;
  for (const Message &x : m) out += "<|im_start|>" + x.role + "\n" + x.content + "<|im_end|>\n";
  if (add_generation_prompt) out += "<|im_start|>assistant\n";
  return out;
}

}  // namespace text
}  // namespace pk

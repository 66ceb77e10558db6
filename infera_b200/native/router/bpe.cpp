// Byte-level BPE tokenizer from a HuggingFace tokenizer.json, restated in
// C++ so the router hashes text prompts into the same token ids the engine
// computes (the engine encodes with the `tokenizers` library,
// add_special_tokens=False).
//
// Supported files (the GPT-2 / Llama-3 / Qwen2 families):
//   model          BPE (merges as "a b" strings or [a, b] pairs; optional
//                  ignore_merges; no dropout, byte fallback or subword affixes)
//   pre_tokenizer  ByteLevel(use_regex=true), or Sequence[Split(regex,
//                  Isolated), ByteLevel(use_regex=false)] where the regex is
//                  one of the three split patterns those families ship
//   normalizer     none, or NFC (a text containing any code point that can
//                  change under NFC is refused: the router then routes it
//                  without locality rather than hash other ids)
//   added_tokens   matched literally before pre-tokenization
// Anything else is refused at load time with a message.
//
// The split patterns are not run through a regex engine: each is a fixed
// ordered alternation, scanned here by hand with the same leftmost-
// alternative, greedy-with-backtracking semantics (lookahead included),
// over Unicode letter / number / White_Space classes from the generated
// tables.
//
// Reference parity: the reference's Rust router tokenizes with the
// `tokenizers` crate (rust/router/src/block_hasher.rs:110-430).
#include <algorithm>
#include <fstream>
#include <mutex>
#include <sstream>
#include <unordered_map>

#include "router.h"
#include "unicode_tables.h"

namespace ib {
namespace {

template <size_t N>
bool in_ranges(const CpRange (&r)[N], uint32_t cp) {
  size_t lo = 0, hi = N;
  while (lo < hi) {
    const size_t mid = (lo + hi) / 2;
    if (cp < r[mid].lo) hi = mid;
    else if (cp > r[mid].hi) lo = mid + 1;
    else return true;
  }
  return false;
}

bool is_letter(uint32_t cp) { return cp < 0x80 ? ((cp | 32) >= 'a' && (cp | 32) <= 'z') : in_ranges(kLetterRanges, cp); }
bool is_number(uint32_t cp) { return cp < 0x80 ? (cp >= '0' && cp <= '9') : in_ranges(kNumberRanges, cp); }
// Unicode White_Space
bool is_space(uint32_t cp) {
  return (cp >= 0x09 && cp <= 0x0D) || cp == 0x20 || cp == 0x85 || cp == 0xA0 || cp == 0x1680 ||
         (cp >= 0x2000 && cp <= 0x200A) || cp == 0x2028 || cp == 0x2029 || cp == 0x202F || cp == 0x205F ||
         cp == 0x3000;
}
bool is_newline(uint32_t cp) { return cp == '\r' || cp == '\n'; }

struct Cp {
  uint32_t cp;
  uint32_t off;  // byte offset in the text
};

// UTF-8 decode; a malformed byte becomes U+FFFD covering that byte
std::vector<Cp> decode_utf8(const std::string& s) {
  std::vector<Cp> out;
  out.reserve(s.size());
  size_t i = 0;
  while (i < s.size()) {
    const unsigned char c = static_cast<unsigned char>(s[i]);
    uint32_t cp = 0xFFFD;
    size_t len = 1;
    if (c < 0x80) {
      cp = c;
    } else if ((c >> 5) == 6 && i + 1 < s.size()) {
      cp = ((c & 0x1F) << 6) | (s[i + 1] & 0x3F);
      len = 2;
    } else if ((c >> 4) == 14 && i + 2 < s.size()) {
      cp = ((c & 0x0F) << 12) | ((s[i + 1] & 0x3F) << 6) | (s[i + 2] & 0x3F);
      len = 3;
    } else if ((c >> 3) == 30 && i + 3 < s.size()) {
      cp = ((c & 0x07) << 18) | ((s[i + 1] & 0x3F) << 12) | ((s[i + 2] & 0x3F) << 6) | (s[i + 3] & 0x3F);
      len = 4;
    }
    out.push_back({cp, static_cast<uint32_t>(i)});
    i += len;
  }
  return out;
}

void append_utf8(std::string* out, uint32_t cp) {
  if (cp < 0x80) {
    out->push_back(static_cast<char>(cp));
  } else if (cp < 0x800) {
    out->push_back(static_cast<char>(0xC0 | (cp >> 6)));
    out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  } else if (cp < 0x10000) {
    out->push_back(static_cast<char>(0xE0 | (cp >> 12)));
    out->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
    out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  } else {
    out->push_back(static_cast<char>(0xF0 | (cp >> 18)));
    out->push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
    out->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
    out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  }
}

enum class SplitMode { kGpt2, kCl100k, kSingleDigit };

// The split patterns of the three families (as they read after JSON decoding).
const char* const kPatGpt2 = R"('s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+)";
const char* const kPatCl100k =
    R"((?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}| ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+)";
const char* const kPatSingleDigit =
    R"((?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+)";

// end (exclusive, in code points) of the pattern's match at i; every
// position matches one of the alternatives, so the result is > i
size_t match_at(const std::vector<Cp>& c, size_t i, SplitMode mode) {
  const size_t n = c.size();
  auto L = [&](size_t k) { return k < n && is_letter(c[k].cp); };
  auto N = [&](size_t k) { return k < n && is_number(c[k].cp); };
  auto S = [&](size_t k) { return k < n && is_space(c[k].cp); };
  auto P = [&](size_t k) { return k < n && !is_space(c[k].cp) && !is_letter(c[k].cp) && !is_number(c[k].cp); };
  // contractions: 's 't 're 've 'm 'll 'd (case-insensitive except GPT-2)
  if (c[i].cp == '\'' && i + 1 < n) {
    const bool fold = mode != SplitMode::kGpt2;
    auto ch = [&](size_t k, char want) {
      if (k >= n) return false;
      uint32_t v = c[k].cp;
      if (fold && v >= 'A' && v <= 'Z') v += 32;
      return v == static_cast<uint32_t>(want);
    };
    if (ch(i + 1, 's') || ch(i + 1, 't') || ch(i + 1, 'm') || ch(i + 1, 'd')) return i + 2;
    if ((ch(i + 1, 'r') && ch(i + 2, 'e')) || (ch(i + 1, 'v') && ch(i + 2, 'e')) ||
        (ch(i + 1, 'l') && ch(i + 2, 'l')))
      return i + 3;
  }
  auto run = [&](size_t k, auto pred) {
    while (pred(k)) ++k;
    return k;
  };
  if (mode == SplitMode::kGpt2) {
    if (c[i].cp == ' ' && L(i + 1)) return run(i + 1, L);
    if (L(i)) return run(i, L);
    if (c[i].cp == ' ' && N(i + 1)) return run(i + 1, N);
    if (N(i)) return run(i, N);
    if (c[i].cp == ' ' && P(i + 1)) return run(i + 1, P);
    if (P(i)) return run(i, P);
  } else {
    // [^\r\n\p{L}\p{N}]?\p{L}+
    if (!is_newline(c[i].cp) && !L(i) && !N(i) && L(i + 1)) return run(i + 1, L);
    if (L(i)) return run(i, L);
    // \p{N}{1,3} or \p{N}
    if (N(i)) {
      const size_t cap = mode == SplitMode::kCl100k ? 3 : 1;
      size_t k = i;
      while (N(k) && k - i < cap) ++k;
      return k;
    }
    // " ?[^\s\p{L}\p{N}]+[\r\n]*"
    {
      size_t k = i;
      if (c[k].cp == ' ' && P(k + 1)) ++k;
      if (P(k)) {
        k = run(k, P);
        while (k < n && is_newline(c[k].cp)) ++k;
        return k;
      }
    }
    // \s*[\r\n]+ : the whitespace run up to its last line break
    if (S(i)) {
      const size_t w = run(i, S);
      for (size_t k = w; k > i; --k)
        if (is_newline(c[k - 1].cp)) return k;
    }
  }
  // \s+(?!\S) then \s+
  if (S(i)) {
    const size_t w = run(i, S);
    if (w == n || w - i == 1) return w;
    return w - 1;
  }
  return i + 1;  // not reached for valid classes; keeps progress
}

// GPT-2 byte-to-unicode map: printable Latin-1 bytes map to themselves, the
// rest to 256 + their order
std::vector<std::string> byte_level_map() {
  std::vector<uint32_t> cps(256, 0);
  std::vector<bool> direct(256, false);
  for (int b = '!'; b <= '~'; ++b) direct[b] = true;
  for (int b = 0xA1; b <= 0xAC; ++b) direct[b] = true;
  for (int b = 0xAE; b <= 0xFF; ++b) direct[b] = true;
  uint32_t extra = 0;
  for (int b = 0; b < 256; ++b) cps[b] = direct[b] ? static_cast<uint32_t>(b) : 256 + extra++;
  std::vector<std::string> out(256);
  for (int b = 0; b < 256; ++b) append_utf8(&out[b], cps[b]);
  return out;
}

class BpeTok : public Tokenizer {
 public:
  std::unordered_map<std::string, uint32_t> vocab;
  std::unordered_map<uint64_t, std::pair<uint32_t, uint32_t>> merges;  // (a, b) -> (rank, merged id)
  std::vector<std::pair<std::string, uint32_t>> added;                 // longest first
  bool added_first[256] = {};                                          // first bytes of added tokens
  std::vector<std::string> byte_map = byte_level_map();
  uint32_t byte_id[256] = {};
  SplitMode mode = SplitMode::kGpt2;
  bool nfc = false;
  bool ignore_merges = false;
  bool prefix_space = false;

  bool try_encode(const std::string& text, std::vector<uint32_t>* out) const override {
    out->clear();
    size_t seg = 0, i = 0;
    while (i < text.size()) {
      if (!added_first[static_cast<unsigned char>(text[i])]) {
        ++i;
        continue;
      }
      size_t hit_len = 0;
      uint32_t hit_id = 0;
      for (const auto& a : added) {
        if (a.first.size() <= text.size() - i && text[i] == a.first[0] &&
            text.compare(i, a.first.size(), a.first) == 0) {
          hit_len = a.first.size();
          hit_id = a.second;
          break;
        }
      }
      if (hit_len == 0) {
        ++i;
        continue;
      }
      if (i > seg && !encode_segment(text.substr(seg, i - seg), out)) return false;
      out->push_back(hit_id);
      i += hit_len;
      seg = i;
    }
    if (seg < text.size() && !encode_segment(text.substr(seg), out)) return false;
    return true;
  }
  std::vector<uint32_t> encode(const std::string& text) const override {
    std::vector<uint32_t> ids;
    try_encode(text, &ids);
    return ids;
  }
  // the engine's chat rendering: "<|role|>\n" + text + "\n" per message,
  // then "<|assistant|>\n", encoded as one text
  bool try_chat(const Value& messages, std::vector<uint32_t>* out) const override {
    std::string text;
    for (const auto& m : messages.arr()) {
      const Value* role = m.get("role");
      text += "<|" + (role && role->is_str() ? role->s : std::string("user")) + "|>\n";
      text += chat_content_text(m.get("content")) + "\n";
    }
    text += "<|assistant|>\n";
    return try_encode(text, out);
  }
  std::vector<uint32_t> chat(const Value& messages) const override {
    std::vector<uint32_t> ids;
    try_chat(messages, &ids);
    return ids;
  }

 private:
  mutable std::mutex mu_;
  mutable std::unordered_map<std::string, std::vector<uint32_t>> cache_;

  bool encode_segment(const std::string& seg_in, std::vector<uint32_t>* out) const {
    std::string seg = seg_in;
    if (prefix_space && (seg.empty() || seg[0] != ' ')) seg.insert(seg.begin(), ' ');
    const auto cps = decode_utf8(seg);
    if (nfc)
      for (const auto& c : cps)
        if (c.cp >= 0x300 && in_ranges(kNfcSensitiveRanges, c.cp)) return false;
    size_t i = 0;
    while (i < cps.size()) {
      const size_t j = match_at(cps, i, mode);
      const size_t b0 = cps[i].off, b1 = j < cps.size() ? cps[j].off : seg.size();
      word(seg.substr(b0, b1 - b0), out);
      i = j;
    }
    return true;
  }

  void word(const std::string& w, std::vector<uint32_t>* out) const {
    {
      std::lock_guard<std::mutex> g(mu_);
      auto it = cache_.find(w);
      if (it != cache_.end()) {
        out->insert(out->end(), it->second.begin(), it->second.end());
        return;
      }
    }
    std::vector<uint32_t> ids;
    std::string mapped;
    for (unsigned char b : w) mapped += byte_map[b];
    auto whole = ignore_merges ? vocab.find(mapped) : vocab.end();
    if (whole != vocab.end()) {
      ids.push_back(whole->second);
    } else {
      ids.reserve(w.size());
      for (unsigned char b : w) ids.push_back(byte_id[b]);
      // merge the lowest-ranked adjacent pair (leftmost among equals) until none is left
      while (ids.size() > 1) {
        uint32_t best = UINT32_MAX, best_id = 0;
        size_t at = 0;
        for (size_t k = 0; k + 1 < ids.size(); ++k) {
          auto it = merges.find((static_cast<uint64_t>(ids[k]) << 32) | ids[k + 1]);
          if (it != merges.end() && it->second.first < best) {
            best = it->second.first;
            best_id = it->second.second;
            at = k;
          }
        }
        if (best == UINT32_MAX) break;
        ids[at] = best_id;
        ids.erase(ids.begin() + static_cast<long>(at) + 1);
      }
    }
    out->insert(out->end(), ids.begin(), ids.end());
    std::lock_guard<std::mutex> g(mu_);
    if (cache_.size() > 200000) cache_.clear();
    cache_.emplace(w, std::move(ids));
  }
};

bool json_bool(const Value* v, bool dflt) { return v && v->is_bool() ? v->b : dflt; }
bool json_nullish(const Value* v) { return !v || v->is_null() || (v->is_str() && v->s.empty()); }

}  // namespace

std::string chat_content_text(const Value* c) {
  if (!c || c->is_null()) return "";
  if (c->is_str()) return c->s;
  if (c->is_arr()) {
    std::string out;
    for (const auto& b : c->arr()) {
      if (b.is_str()) out += b.s;
      else if (b.is_obj()) {
        const Value* t = b.get("type");
        if (t && t->is_str() && (t->s == "text" || t->s == "input_text")) {
          const Value* x = b.get("text");
          if (x && x->is_str()) out += x->s;
        }
      }
    }
    return out;
  }
  return dump_json(*c);
}

std::unique_ptr<Tokenizer> load_bpe_tokenizer(const Value& v, std::string* err) {
  const Value* model = v.get("model");
  auto tok = std::make_unique<BpeTok>();
  if (!json_nullish(model->get("dropout")) || json_bool(model->get("byte_fallback"), false) ||
      !json_nullish(model->get("continuing_subword_prefix")) || !json_nullish(model->get("end_of_word_suffix"))) {
    *err = "BPE with dropout, byte fallback or subword affixes is not supported";
    return nullptr;
  }
  tok->ignore_merges = json_bool(model->get("ignore_merges"), false);
  if (const Value* voc = model->get("vocab"); voc && voc->is_obj())
    for (const auto& kv : voc->obj()) tok->vocab[kv.first] = static_cast<uint32_t>(kv.second.as_int());
  for (int b = 0; b < 256; ++b) {
    auto it = tok->vocab.find(tok->byte_map[b]);
    if (it == tok->vocab.end()) {
      *err = "vocabulary lacks the byte-level alphabet";
      return nullptr;
    }
    tok->byte_id[b] = it->second;
  }
  if (const Value* m = model->get("merges"); m && m->is_arr()) {
    uint32_t rank = 0;
    for (const auto& e : m->arr()) {
      std::string a, b;
      if (e.is_str()) {
        const size_t sp = e.s.find(' ');
        if (sp == std::string::npos) continue;
        a = e.s.substr(0, sp);
        b = e.s.substr(sp + 1);
      } else if (e.is_arr() && e.arr().size() == 2 && e.arr()[0].is_str() && e.arr()[1].is_str()) {
        a = e.arr()[0].s;
        b = e.arr()[1].s;
      } else {
        continue;
      }
      auto ia = tok->vocab.find(a), ib = tok->vocab.find(b), im = tok->vocab.find(a + b);
      if (ia != tok->vocab.end() && ib != tok->vocab.end() && im != tok->vocab.end())
        tok->merges.emplace((static_cast<uint64_t>(ia->second) << 32) | ib->second, std::make_pair(rank, im->second));
      ++rank;
    }
  }
  // normalizer
  const Value* norm = v.get("normalizer");
  if (norm && !norm->is_null()) {
    const Value* t = norm->get("type");
    if (t && t->is_str() && t->s == "NFC") {
      tok->nfc = true;
    } else {
      *err = "normalizer " + (t && t->is_str() ? t->s : std::string("?")) + " is not supported";
      return nullptr;
    }
  }
  // pre-tokenizer
  const Value* pre = v.get("pre_tokenizer");
  const Value* ptype = pre ? pre->get("type") : nullptr;
  if (ptype && ptype->is_str() && ptype->s == "ByteLevel") {
    if (!json_bool(pre->get("use_regex"), true)) {
      *err = "ByteLevel without a split pattern is not supported";
      return nullptr;
    }
    tok->mode = SplitMode::kGpt2;
    tok->prefix_space = json_bool(pre->get("add_prefix_space"), false);
  } else if (ptype && ptype->is_str() && ptype->s == "Sequence") {
    const Value* list = pre->get("pretokenizers");
    bool ok = list && list->is_arr() && list->arr().size() == 2;
    if (ok) {
      const Value& sp = list->arr()[0];
      const Value& bl = list->arr()[1];
      const Value* st = sp.get("type");
      const Value* pat = sp.get("pattern");
      const Value* rx = pat ? pat->get("Regex") : nullptr;
      const Value* beh = sp.get("behavior");
      const Value* bt = bl.get("type");
      ok = st && st->is_str() && st->s == "Split" && rx && rx->is_str() && beh && beh->is_str() &&
           beh->s == "Isolated" && !json_bool(sp.get("invert"), false) && bt && bt->is_str() &&
           bt->s == "ByteLevel" && !json_bool(bl.get("use_regex"), true) &&
           !json_bool(bl.get("add_prefix_space"), false);
      if (ok) {
        if (rx->s == kPatCl100k) tok->mode = SplitMode::kCl100k;
        else if (rx->s == kPatSingleDigit) tok->mode = SplitMode::kSingleDigit;
        else if (rx->s == kPatGpt2) tok->mode = SplitMode::kGpt2;
        else ok = false;
      }
    }
    if (!ok) {
      *err = "pre-tokenizer sequence is not Split(<known pattern>) + ByteLevel";
      return nullptr;
    }
  } else {
    *err = "pre-tokenizer " + (ptype && ptype->is_str() ? ptype->s : std::string("none")) + " is not supported";
    return nullptr;
  }
  if (const Value* at = v.get("added_tokens"); at && at->is_arr())
    for (const auto& a : at->arr()) {
      const Value* c = a.get("content");
      const Value* id = a.get("id");
      if (c && c->is_str() && !c->s.empty() && id) {
        tok->added.emplace_back(c->s, static_cast<uint32_t>(id->as_int()));
        tok->added_first[static_cast<unsigned char>(c->s[0])] = true;
      }
    }
  std::stable_sort(tok->added.begin(), tok->added.end(),
                   [](const auto& x, const auto& y) { return x.first.size() > y.first.size(); });
  return tok;
}

}  // namespace ib

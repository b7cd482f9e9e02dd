// BpeTokenizer (src/tokenizer.rs:148-600): the text step before the token
// loop, on the host in C++ so the reference's Rust host can bind it through
// the C ABI like the rest of the path.
//
//   * pre-tokenisation: the reference's pattern
//     's|'t|'re|'ve|'m|'ll|'d| ?[^\s]+|\s+ with leftmost-first alternation
//     and Unicode White_Space for \s, scanned by hand (no regex engine);
//   * BPE per piece: start from the piece's characters, repeatedly merge
//     every occurrence of the adjacent pair with the lowest rank (first pair
//     on ties), ranks keyed by the two tokens' ids (src/tokenizer.rs:456-512);
//   * pieces missing from the vocabulary fall back to their UTF-8 bytes
//     through the <0xNN> byte tokens (id 0 where none exists);
//   * decode: token texts concatenated, a <0xNN> token becoming the character
//     U+00NN (the reference pushes `byte as char`).
//
// Where the reference leaves the result open, this code fixes one:
//   * encode_with_special orders special tokens found at the same position
//     longest first (the reference's order comes from a HashMap walk), and
//     skips a special occurrence that overlaps the previous one (the
//     reference would slice its text backwards and panic);
//   * an empty special-token text is never searched (the reference's search
//     would not advance).
#include <algorithm>
#include <cstring>
#include <map>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/fishai_cuda.h"
#include "fa_host.hpp"
#include "gguf.hpp"
#include <new>

namespace fa {

namespace {

enum : int32_t { kNormal = 0, kUnknown = 1, kByte = 2, kControl = 3, kUserDefined = 4 };

// TokenType::from (src/tokenizer.rs:55-66): unknown values -> Unknown
int32_t token_type_from(int32_t v) { return (v >= 0 && v <= 4) ? v : kUnknown; }

// Unicode White_Space (the \s class of the reference's regex)
bool is_space(uint32_t c) {
  return (c >= 0x09 && c <= 0x0D) || c == 0x20 || c == 0x85 || c == 0xA0 || c == 0x1680 ||
         (c >= 0x2000 && c <= 0x200A) || c == 0x2028 || c == 0x2029 || c == 0x202F || c == 0x205F || c == 0x3000;
}

// one code point of UTF-8 text at byte i: (code point, byte length); invalid
// bytes stand for themselves (the reference's &str is valid UTF-8 already)
std::pair<uint32_t, size_t> utf8_at(const std::string &s, size_t i) {
  const uint8_t b = (uint8_t)s[i];
  auto cont = [&](size_t k) { return i + k < s.size() && ((uint8_t)s[i + k] & 0xC0) == 0x80; };
  if (b < 0x80) return {b, 1};
  if ((b & 0xE0) == 0xC0 && cont(1)) return {((b & 0x1Fu) << 6) | ((uint8_t)s[i + 1] & 0x3Fu), 2};
  if ((b & 0xF0) == 0xE0 && cont(1) && cont(2))
    return {((b & 0x0Fu) << 12) | (((uint8_t)s[i + 1] & 0x3Fu) << 6) | ((uint8_t)s[i + 2] & 0x3Fu), 3};
  if ((b & 0xF8) == 0xF0 && cont(1) && cont(2) && cont(3))
    return {((b & 0x07u) << 18) | (((uint8_t)s[i + 1] & 0x3Fu) << 12) | (((uint8_t)s[i + 2] & 0x3Fu) << 6) |
                ((uint8_t)s[i + 3] & 0x3Fu),
            4};
  return {b, 1};
}

void utf8_put(std::string &out, uint32_t c) {
  if (c < 0x80) {
    out += (char)c;
  } else if (c < 0x800) {
    out += (char)(0xC0 | (c >> 6));
    out += (char)(0x80 | (c & 0x3F));
  } else if (c < 0x10000) {
    out += (char)(0xE0 | (c >> 12));
    out += (char)(0x80 | ((c >> 6) & 0x3F));
    out += (char)(0x80 | (c & 0x3F));
  } else {
    out += (char)(0xF0 | (c >> 18));
    out += (char)(0x80 | ((c >> 12) & 0x3F));
    out += (char)(0x80 | ((c >> 6) & 0x3F));
    out += (char)(0x80 | (c & 0x3F));
  }
}

// parse_byte_token_text (src/tokenizer.rs:556-563): "<0xNN>" -> NN
int byte_token_value(const std::string &t) {
  if (t.size() != 6 || t.compare(0, 3, "<0x") != 0 || t[5] != '>') return -1;
  int v = 0;
  for (int k = 3; k < 5; ++k) {
    const char c = t[k];
    const int d = (c >= '0' && c <= '9') ? c - '0' : (c >= 'a' && c <= 'f') ? c - 'a' + 10
                  : (c >= 'A' && c <= 'F') ? c - 'A' + 10 : -1;
    if (d < 0) return -1;
    v = v * 16 + d;
  }
  return v;
}

}  // namespace

struct Tokenizer {
  std::vector<std::string> text;
  std::vector<float> score;
  std::vector<int32_t> type;
  std::unordered_map<std::string, uint32_t> to_id;
  std::vector<uint32_t> byte_tokens = std::vector<uint32_t>(256, 0);
  std::map<std::pair<uint32_t, uint32_t>, uint32_t> ranks;
  std::vector<std::pair<std::string, uint32_t>> specials;
  fa_tokenizer_config cfg{};

  // BpeTokenizer::from_gguf (src/tokenizer.rs:202-286)
  void build(const std::vector<std::string> &texts, const std::vector<float> &scores,
             const std::vector<int32_t> &types, const std::string *merges) {
    const size_t n = texts.size();
    text = texts;
    score.assign(n, 0.0f);
    type.assign(n, kNormal);
    bool byte_set = false;
    std::unordered_map<std::string, uint32_t> special_map;
    for (size_t i = 0; i < n; ++i) {
      if (i < scores.size()) score[i] = scores[i];
      if (i < types.size()) type[i] = token_type_from(types[i]);
      if (type[i] == kByte) {
        const int b = byte_token_value(text[i]);
        if (b >= 0) {
          byte_tokens[b] = (uint32_t)i;
          byte_set = true;
        }
      }
      if (type[i] == kControl || type[i] == kUserDefined) special_map[text[i]] = (uint32_t)i;
      to_id[text[i]] = (uint32_t)i;  // a later duplicate text wins, as HashMap::insert
    }
    if (!byte_set)  // build_byte_tokens_fallback (src/tokenizer.rs:566-573)
      for (size_t i = 0; i < n; ++i) {
        const int b = byte_token_value(text[i]);
        if (b >= 0) byte_tokens[b] = (uint32_t)i;
      }
    for (auto &kv : special_map)
      if (!kv.first.empty()) specials.push_back(kv);
    if (merges) {  // rank = line index among all lines (src/tokenizer.rs:256-274)
      size_t rank = 0, pos = 0;
      while (pos <= merges->size()) {
        size_t e = merges->find('\n', pos);
        if (e == std::string::npos) e = merges->size();
        std::string line = merges->substr(pos, e - pos);
        if (!line.empty() && line.back() == '\r') line.pop_back();  // str::lines drops "\r\n"
        const size_t a = line.find_first_not_of(" \t\n\r\f\v"), b = line.find_last_not_of(" \t\n\r\f\v");
        line = a == std::string::npos ? std::string() : line.substr(a, b - a + 1);
        if (!line.empty() && line[0] != '#') {
          const size_t sp = line.find(' ');
          if (sp != std::string::npos) {
            const std::string l = line.substr(0, sp);
            const size_t sp2 = line.find(' ', sp + 1);
            const std::string r = line.substr(sp + 1, sp2 == std::string::npos ? std::string::npos : sp2 - sp - 1);
            auto li = to_id.find(l), ri = to_id.find(r);
            if (li != to_id.end() && ri != to_id.end()) ranks[{li->second, ri->second}] = (uint32_t)rank;
          }
        }
        ++rank;
        if (e >= merges->size()) break;
        pos = e + 1;
      }
    }
  }

  // the reference's pre-tokenizer pattern, leftmost-first
  std::vector<std::string> pieces(const std::string &s) const {
    std::vector<std::string> out;
    static const char *kContractions[7] = {"'s", "'t", "'re", "'ve", "'m", "'ll", "'d"};
    size_t i = 0;
    while (i < s.size()) {
      bool done = false;
      for (const char *c : kContractions) {
        const size_t n = std::strlen(c);
        if (s.compare(i, n, c) == 0) {
          out.push_back(s.substr(i, n));
          i += n;
          done = true;
          break;
        }
      }
      if (done) continue;
      auto [c0, l0] = utf8_at(s, i);
      size_t j = i;
      if (c0 == ' ' && i + 1 < s.size() && !is_space(utf8_at(s, i + 1).first)) j = i + 1;  //  ?[^\s]+ with the space
      if (!is_space(utf8_at(s, j).first)) {
        while (j < s.size()) {
          auto [c, l] = utf8_at(s, j);
          if (is_space(c)) break;
          j += l;
        }
      } else {  // \s+
        j = i;
        while (j < s.size()) {
          auto [c, l] = utf8_at(s, j);
          if (!is_space(c)) break;
          j += l;
        }
      }
      (void)l0;
      out.push_back(s.substr(i, j - i));
      i = j;
    }
    return out;
  }

  // BpeTokenizer::bpe (src/tokenizer.rs:456-512)
  std::vector<std::string> bpe(const std::string &piece) const {
    std::vector<std::string> w;
    for (size_t i = 0; i < piece.size();) {
      const size_t l = utf8_at(piece, i).second;
      w.push_back(piece.substr(i, l));
      i += l;
    }
    while (w.size() > 1) {
      int best = -1;
      uint32_t best_rank = UINT32_MAX;
      for (size_t i = 0; i + 1 < w.size(); ++i) {
        auto li = to_id.find(w[i]), ri = to_id.find(w[i + 1]);
        if (li == to_id.end() || ri == to_id.end()) continue;
        auto it = ranks.find({li->second, ri->second});
        if (it != ranks.end() && it->second < best_rank) {
          best_rank = it->second;
          best = (int)i;
        }
      }
      if (best < 0) break;
      const std::string a = w[best], b = w[best + 1];
      std::vector<std::string> nw;
      for (size_t i = 0; i < w.size();) {
        if (i + 1 < w.size() && w[i] == a && w[i + 1] == b) {
          nw.push_back(a + b);
          i += 2;
        } else {
          nw.push_back(w[i]);
          i += 1;
        }
      }
      w.swap(nw);
    }
    return w;
  }

  // BpeTokenizer::encode (src/tokenizer.rs:290-344)
  void encode(const std::string &text_in, bool add_special, std::vector<uint32_t> &ids) const {
    if (add_special && cfg.prepend_bos && cfg.bos_token_id >= 0) ids.push_back((uint32_t)cfg.bos_token_id);
    std::string s = text_in;
    if (cfg.add_space_prefix && !s.empty() && s[0] != ' ') s = " " + s;
    if (cfg.remove_special_whitespaces) {  // src/tokenizer.rs:576-583
      std::string o;
      for (size_t i = 0; i < s.size();) {
        auto [c, l] = utf8_at(s, i);
        if (c == 0xA0 || c == 0x200B || c == 0x200C || c == 0x200D || c == 0xFEFF) o += ' ';
        else o.append(s, i, l);
        i += l;
      }
      s.swap(o);
    }
    for (const std::string &p : pieces(s))
      for (const std::string &sw : bpe(p)) {
        auto it = to_id.find(sw);
        if (it != to_id.end()) {
          ids.push_back(it->second);
        } else {
          for (unsigned char b : sw) ids.push_back(byte_tokens[b]);
        }
      }
    if (add_special && cfg.add_eos && cfg.eos_token_id >= 0) ids.push_back((uint32_t)cfg.eos_token_id);
  }

  // BpeTokenizer::encode_with_special (src/tokenizer.rs:347-391)
  void encode_with_special(const std::string &s, std::vector<uint32_t> &ids) const {
    struct Hit {
      size_t pos, len;
      uint32_t id;
    };
    std::vector<Hit> hits;
    for (const auto &sp : specials)
      for (size_t from = 0;;) {
        const size_t p = s.find(sp.first, from);
        if (p == std::string::npos) break;
        hits.push_back({p, sp.first.size(), sp.second});
        from = p + sp.first.size();
      }
    std::sort(hits.begin(), hits.end(), [](const Hit &a, const Hit &b) {
      return a.pos != b.pos ? a.pos < b.pos : a.len != b.len ? a.len > b.len : a.id < b.id;
    });
    size_t last = 0;
    for (const Hit &h : hits) {
      if (h.pos < last) continue;
      if (h.pos > last) encode(s.substr(last, h.pos - last), false, ids);
      ids.push_back(h.id);
      last = h.pos + h.len;
    }
    if (last < s.size()) encode(s.substr(last), false, ids);
  }

  // BpeTokenizer::decode (src/tokenizer.rs:394-408)
  std::string decode(const uint32_t *ids, size_t n) const {
    std::string out;
    for (size_t i = 0; i < n; ++i) {
      if (ids[i] >= text.size()) continue;
      const int b = byte_token_value(text[ids[i]]);
      if (b >= 0) utf8_put(out, (uint32_t)b);
      else out += text[ids[i]];
    }
    return out;
  }
};

}  // namespace fa

using fa::Tokenizer;
struct fa_tokenizer {
  Tokenizer t;
};

namespace fa {
// the tokenizer a GGUF file carries (tokenizer.ggml.tokens / scores /
// token_type / merges and the config keys of
// parse_tokenizer_config_from_gguf, src/tokenizer.rs:520-553)
int tokenizer_from_gguf(const Gguf &g, fa_tokenizer **out) {
  const std::vector<std::string> *tokens = g.meta_str_array("tokenizer.ggml.tokens");
  if (!tokens) return fail(FA_ERR_GGUF, "GGUF has no tokenizer.ggml.tokens array");
  std::vector<float> scores;
  std::vector<int32_t> types;
  if (const std::vector<double> *v = g.meta_num_array("tokenizer.ggml.scores"))
    for (double x : *v) scores.push_back((float)x);
  if (const std::vector<double> *v = g.meta_num_array("tokenizer.ggml.token_type"))
    for (double x : *v) types.push_back((int32_t)x);
  std::string merges;
  const std::vector<std::string> *ml = g.meta_str_array("tokenizer.ggml.merges");
  if (ml)
    for (size_t i = 0; i < ml->size(); ++i) merges += (i ? "\n" : "") + (*ml)[i];
  fa_tokenizer *t = new (std::nothrow) fa_tokenizer();
  if (!t) return fail(FA_ERR_OOM, "out of memory");
  fa_tokenizer_config &c = t->t.cfg;
  fa_tokenizer_config_default(&c);
  uint64_t u;
  bool b;
  if (g.meta_u64("tokenizer.ggml.bos_token_id", &u)) c.bos_token_id = (int64_t)u;
  if (g.meta_u64("tokenizer.ggml.eos_token_id", &u)) c.eos_token_id = (int64_t)u;
  if (g.meta_u64("tokenizer.ggml.eot_token_id", &u)) c.eot_token_id = (int64_t)u;
  if (g.meta_u64("tokenizer.ggml.eom_token_id", &u)) c.eom_token_id = (int64_t)u;
  if (g.meta_u64("tokenizer.ggml.unknown_token_id", &u)) c.unk_token_id = (int64_t)u;
  c.add_bos = g.meta_bool("tokenizer.ggml.add_bos", &b) && b;
  c.add_eos = g.meta_bool("tokenizer.ggml.add_eos", &b) && b;
  c.add_space_prefix = g.meta_bool("tokenizer.ggml.add_space_prefix", &b) && b;
  c.remove_special_whitespaces = g.meta_bool("tokenizer.ggml.remove_special_whitespaces", &b) && b;
  c.prepend_bos = g.meta_bool("tokenizer.ggml.prepend_bos", &b) && b;
  t->t.build(*tokens, scores, types, ml ? &merges : nullptr);
  *out = t;
  return FA_OK;
}
}  // namespace fa

namespace {
int copy_ids(const std::vector<uint32_t> &v, uint32_t *ids, size_t cap, size_t *n) {
  *n = v.size();
  if (ids) std::memcpy(ids, v.data(), std::min(cap, v.size()) * sizeof(uint32_t));
  return FA_OK;
}
}  // namespace

extern "C" {

void fa_tokenizer_config_default(fa_tokenizer_config *c) {
  if (!c) return;
  std::memset(c, 0, sizeof *c);
  c->bos_token_id = c->eos_token_id = c->eot_token_id = c->eom_token_id = c->unk_token_id = -1;
}

int fa_tokenizer_create(const char *const *texts, uint32_t n_tokens, const float *scores, uint32_t n_scores,
                        const int32_t *types, uint32_t n_types, const char *merges, const fa_tokenizer_config *cfg,
                        fa_tokenizer **out) {
  if (!out || (n_tokens && !texts)) return fa::fail(FA_ERR_INVALID, "fa_tokenizer_create: null argument");
  fa_tokenizer *t = new (std::nothrow) fa_tokenizer();
  if (!t) return fa::fail(FA_ERR_OOM, "out of memory");
  std::vector<std::string> tx(n_tokens);
  for (uint32_t i = 0; i < n_tokens; ++i) tx[i] = texts[i] ? texts[i] : "";
  std::vector<float> sc(scores ? scores : nullptr, scores ? scores + n_scores : nullptr);
  std::vector<int32_t> ty(types ? types : nullptr, types ? types + n_types : nullptr);
  if (cfg) t->t.cfg = *cfg;
  else fa_tokenizer_config_default(&t->t.cfg);
  std::string m = merges ? merges : "";
  t->t.build(tx, sc, ty, merges ? &m : nullptr);
  *out = t;
  return FA_OK;
}

void fa_tokenizer_free(fa_tokenizer *t) { delete t; }

int fa_tokenizer_encode(const fa_tokenizer *t, const char *text, size_t len, int32_t add_special,
                        int32_t with_special, uint32_t *ids, size_t cap, size_t *n) {
  if (!t || !n || (len && !text)) return fa::fail(FA_ERR_INVALID, "fa_tokenizer_encode: null argument");
  const std::string s(text ? text : "", len);
  std::vector<uint32_t> v;
  if (with_special) t->t.encode_with_special(s, v);
  else t->t.encode(s, add_special != 0, v);
  return copy_ids(v, ids, cap, n);
}

int fa_tokenizer_decode(const fa_tokenizer *t, const uint32_t *ids, size_t n, char *buf, size_t cap, size_t *len) {
  if (!t || !len || (n && !ids)) return fa::fail(FA_ERR_INVALID, "fa_tokenizer_decode: null argument");
  const std::string s = t->t.decode(ids, n);
  *len = s.size();
  if (buf && cap) {
    const size_t k = std::min(cap - 1, s.size());
    std::memcpy(buf, s.data(), k);
    buf[k] = 0;
  }
  return FA_OK;
}

int fa_tokenizer_info(const fa_tokenizer *t, uint32_t *vocab_size, fa_tokenizer_config *cfg) {
  if (!t) return fa::fail(FA_ERR_INVALID, "fa_tokenizer_info: null argument");
  if (vocab_size) *vocab_size = (uint32_t)t->t.text.size();
  if (cfg) *cfg = t->t.cfg;
  return FA_OK;
}

int fa_tokenizer_piece(const fa_tokenizer *t, uint32_t id, char *buf, size_t cap, size_t *len, int32_t *type) {
  if (!t || !len) return fa::fail(FA_ERR_INVALID, "fa_tokenizer_piece: null argument");
  if (id >= t->t.text.size()) return fa::fail(FA_ERR_INVALID, "token id out of range");
  const std::string &s = t->t.text[id];
  *len = s.size();
  if (type) *type = t->t.type[id];
  if (buf && cap) {
    const size_t k = std::min(cap - 1, s.size());
    std::memcpy(buf, s.data(), k);
    buf[k] = 0;
  }
  return FA_OK;
}

int fa_tokenizer_byte_token(const fa_tokenizer *t, uint32_t byte_value, uint32_t *id) {
  if (!t || !id || byte_value > 255) return fa::fail(FA_ERR_INVALID, "fa_tokenizer_byte_token: bad argument");
  *id = t->t.byte_tokens[byte_value];
  return FA_OK;
}

}  // extern "C"

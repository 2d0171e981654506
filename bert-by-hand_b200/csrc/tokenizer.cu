// WordPiece tokenizer (host): the step before the path. The reference tokenizes with the
// HF tokenizer of the sentence-transformers model (scripts/dump_corpus.py:34-38,
// dump_weights.py:100-106: BERT uncased, truncation to 128, [CLS] ... [SEP]); it has no
// tokenizer of its own. This restates that algorithm in C++ and emits the packed ids and
// cu_seqlens the packed forward takes:
//   1. clean: drop NUL, U+FFFD and control characters; whitespace -> ' '
//   2. put spaces around CJK ideographs
//   3. (uncased) canonical decomposition of accented letters, drop combining marks (Mn),
//      lowercase
//   4. split on whitespace; every punctuation character is a token of its own
//   5. WordPiece: greedy longest match, continuation pieces prefixed "##"; a word longer
//      than 100 characters, or one with an unmatched piece, becomes [UNK]
//   6. [CLS] + pieces + [SEP], pieces truncated to max_len - 2
// Large batches are split over host threads (contiguous ranges, output in text order).
// Character classes, decompositions and case mappings cover all of Unicode (tables in
// unicode_tables.h, generated from the Unicode 15.0 character database).
#include "internal.h"
#include "unicode_tables.h"
#include "../../include/bbh.h"

#include <cstdint>
#include <cstdio>
#include <algorithm>
#include <cstring>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

struct bbh_vocab {
  std::unordered_map<std::string, int32_t> ids;
  bool lower = true;
  int32_t unk = -1, cls = -1, sep = -1;
};

namespace {

// ---------------------------------------------------------------- UTF-8
void utf8_decode(const char* s, std::vector<uint32_t>* out) {
  out->clear();
  const auto* p = reinterpret_cast<const uint8_t*>(s);
  while (*p) {
    uint32_t c = *p, need = 0;
    if (c < 0x80) {
      need = 0;
    } else if ((c & 0xE0) == 0xC0) {
      c &= 0x1F, need = 1;
    } else if ((c & 0xF0) == 0xE0) {
      c &= 0x0F, need = 2;
    } else if ((c & 0xF8) == 0xF0) {
      c &= 0x07, need = 3;
    } else {
      out->push_back(0xFFFD);  // stray continuation or invalid lead byte
      ++p;
      continue;
    }
    ++p;
    bool ok = true;
    for (uint32_t k = 0; k < need; ++k, ++p) {
      if ((*p & 0xC0) != 0x80) {
        ok = false;
        break;
      }
      c = (c << 6) | (*p & 0x3F);
    }
    out->push_back(ok ? c : 0xFFFD);
  }
}

void utf8_append(uint32_t c, std::string* s) {
  if (c < 0x80) {
    s->push_back(char(c));
  } else if (c < 0x800) {
    s->push_back(char(0xC0 | (c >> 6)));
    s->push_back(char(0x80 | (c & 0x3F)));
  } else if (c < 0x10000) {
    s->push_back(char(0xE0 | (c >> 12)));
    s->push_back(char(0x80 | ((c >> 6) & 0x3F)));
    s->push_back(char(0x80 | (c & 0x3F)));
  } else {
    s->push_back(char(0xF0 | (c >> 18)));
    s->push_back(char(0x80 | ((c >> 12) & 0x3F)));
    s->push_back(char(0x80 | ((c >> 6) & 0x3F)));
    s->push_back(char(0x80 | (c & 0x3F)));
  }
}

// ---------------------------------------------------------------- character classes
// Tables generated from the Unicode character database (gen_unicode_tables.py).
bool in_runs(const uint32_t (*runs)[2], int n, uint32_t c) {
  int lo = 0, hi = n - 1;
  while (lo <= hi) {
    const int mid = (lo + hi) >> 1;
    if (c < runs[mid][0])
      hi = mid - 1;
    else if (c > runs[mid][1])
      lo = mid + 1;
    else
      return true;
  }
  return false;
}

template <typename E>
const E* find_entry(const E* table, int n, uint32_t c) {
  int lo = 0, hi = n - 1;
  while (lo <= hi) {
    const int mid = (lo + hi) >> 1;
    if (c < table[mid].cp)
      hi = mid - 1;
    else if (c > table[mid].cp)
      lo = mid + 1;
    else
      return &table[mid];
  }
  return nullptr;
}

// White_Space property (tab, newline and return count as whitespace, not control)
bool is_whitespace(uint32_t c) {
  return (c >= 0x09 && c <= 0x0D) || c == 0x20 || c == 0x85 || c == 0xA0 || c == 0x1680 ||
         (c >= 0x2000 && c <= 0x200A) || c == 0x2028 || c == 0x2029 || c == 0x202F || c == 0x205F || c == 0x3000;
}
bool is_control(uint32_t c) { return in_runs(bbh_uni::kControl, bbh_uni::kControlRuns, c); }
bool is_punct(uint32_t c) { return in_runs(bbh_uni::kPunct, bbh_uni::kPunctRuns, c); }
bool is_mark(uint32_t c) { return in_runs(bbh_uni::kMark, bbh_uni::kMarkRuns, c); }

bool is_cjk(uint32_t c) {
  return (c >= 0x4E00 && c <= 0x9FFF) || (c >= 0x3400 && c <= 0x4DBF) || (c >= 0x20000 && c <= 0x2A6DF) ||
         (c >= 0x2A700 && c <= 0x2B73F) || (c >= 0x2B740 && c <= 0x2B81F) || (c >= 0x2B820 && c <= 0x2CEAF) ||
         (c >= 0xF900 && c <= 0xFAFF) || (c >= 0x2F800 && c <= 0x2FA1F);
}

// Canonical decomposition without combining marks (accent stripping), appended to out.
void strip_accents(uint32_t c, std::vector<uint32_t>* out) {
  if (c >= 0xAC00 && c <= 0xD7A3) {  // Hangul syllable -> leading, vowel (, trailing) jamo
    const uint32_t s = c - 0xAC00;
    out->push_back(0x1100 + s / (21 * 28));
    out->push_back(0x1161 + (s % (21 * 28)) / 28);
    if (s % 28) out->push_back(0x11A7 + s % 28);
    return;
  }
  if (is_mark(c)) return;
  const auto* e = find_entry(bbh_uni::kDecomp, bbh_uni::kDecompCount, c);
  if (!e) {
    out->push_back(c);
    return;
  }
  for (int k = 0; k < e->n; ++k) out->push_back(e->to[k]);
}

void lower_into(uint32_t c, std::vector<uint32_t>* out) {
  if (c < 0x80) {
    out->push_back(c >= 'A' && c <= 'Z' ? c + 32 : c);
    return;
  }
  const auto* e = find_entry(bbh_uni::kLower, bbh_uni::kLowerCount, c);
  if (!e) {
    out->push_back(c);
    return;
  }
  for (int k = 0; k < e->n; ++k) out->push_back(e->to[k]);
}

// ---------------------------------------------------------------- pipeline
// Normalisation (in the order of BERT's normaliser) and the whitespace / punctuation split.
void normalize_and_split(const bbh_vocab& v, const std::vector<uint32_t>& in, std::vector<std::vector<uint32_t>>* words) {
  words->clear();
  std::vector<uint32_t> cur, a, b;
  auto flush = [&]() {
    if (!cur.empty()) words->push_back(cur);
    cur.clear();
  };
  for (uint32_t c : in) {
    if (c == 0 || c == 0xFFFD || is_control(c)) continue;  // clean
    if (is_whitespace(c)) {
      flush();
      continue;
    }
    a.assign(1, c);
    if (v.lower) {
      b.clear();
      for (uint32_t x : a) strip_accents(x, &b);
      a.clear();
      for (uint32_t x : b) lower_into(x, &a);
    }
    const bool cjk = is_cjk(c);
    for (uint32_t x : a) {
      if (is_whitespace(x)) {
        flush();
      } else if (cjk || is_punct(x)) {
        flush();
        words->push_back({x});
      } else {
        cur.push_back(x);
      }
    }
  }
  flush();
}

void wordpiece(const bbh_vocab& v, const std::vector<uint32_t>& word, std::vector<int32_t>* out) {
  if (word.size() > 100) {
    out->push_back(v.unk);
    return;
  }
  // UTF-8 of every prefix boundary, so substrings are byte ranges
  std::string bytes;
  std::vector<size_t> at(word.size() + 1);
  for (size_t i = 0; i < word.size(); ++i) {
    at[i] = bytes.size();
    utf8_append(word[i], &bytes);
  }
  at[word.size()] = bytes.size();
  std::vector<int32_t> pieces;
  size_t start = 0;
  std::string key;
  while (start < word.size()) {
    size_t end = word.size();
    int32_t found = -1;
    while (end > start) {
      key.assign(start > 0 ? "##" : "");
      key.append(bytes, at[start], at[end] - at[start]);
      auto it = v.ids.find(key);
      if (it != v.ids.end()) {
        found = it->second;
        break;
      }
      --end;
    }
    if (found < 0) {
      out->push_back(v.unk);
      return;
    }
    pieces.push_back(found);
    start = end;
  }
  out->insert(out->end(), pieces.begin(), pieces.end());
}

}  // namespace

extern "C" {

int bbh_vocab_load(const char* path, int lowercase, bbh_vocab** out) {
  if (!path || !out) return bbh::internal_fail(BBH_ERR_ARG, "bbh_vocab_load: bad arguments");
  FILE* f = std::fopen(path, "rb");
  if (!f) return bbh::internal_fail(BBH_ERR_IO, std::string("cannot open ") + path);
  auto* v = new bbh_vocab;
  v->lower = lowercase != 0;
  std::string line;
  int32_t id = 0;
  int ch;
  auto add = [&]() {
    while (!line.empty() && (line.back() == '\r' || line.back() == '\n')) line.pop_back();
    v->ids.emplace(line, id++);  // the first occurrence of a duplicate keeps its id
    line.clear();
  };
  while ((ch = std::fgetc(f)) != EOF) {
    if (ch == '\n')
      add();
    else
      line.push_back(char(ch));
  }
  if (!line.empty()) add();
  std::fclose(f);
  auto find = [&](const char* t) {
    auto it = v->ids.find(t);
    return it == v->ids.end() ? -1 : it->second;
  };
  v->unk = find("[UNK]");
  v->cls = find("[CLS]");
  v->sep = find("[SEP]");
  if (v->unk < 0 || v->cls < 0 || v->sep < 0) {
    delete v;
    return bbh::internal_fail(BBH_ERR_IO, std::string(path) + ": vocabulary lacks [UNK], [CLS] or [SEP]");
  }
  *out = v;
  return BBH_OK;
}

void bbh_vocab_free(bbh_vocab* v) { delete v; }

int bbh_vocab_size(const bbh_vocab* v) { return v ? static_cast<int>(v->ids.size()) : 0; }

int bbh_tokenize(const bbh_vocab* v, const char* const* texts, int n, int max_len, int32_t* ids, int64_t ids_cap,
                 int32_t* cu_seqlens, int64_t* total) {
  if (!v || n < 0 || (n > 0 && !texts) || max_len < 2 || !cu_seqlens || !total || ids_cap < 0 || (ids_cap > 0 && !ids))
    return bbh::internal_fail(BBH_ERR_ARG, "bbh_tokenize: bad arguments");
  for (int i = 0; i < n; ++i)
    if (!texts[i]) return bbh::internal_fail(BBH_ERR_ARG, "bbh_tokenize: null text " + std::to_string(i));
  // Texts are split into contiguous ranges tokenized by host threads into private buffers,
  // then laid out in text order: the result does not depend on the thread count.
  const int hw = static_cast<int>(std::thread::hardware_concurrency());
  const int nthreads = std::max(1, std::min({hw > 0 ? hw : 1, 32, n / 512}));
  std::vector<std::vector<int32_t>> part(static_cast<size_t>(nthreads));
  std::vector<int32_t> lens(static_cast<size_t>(n));
  auto work = [&](int t) {
    const int lo = int(int64_t(n) * t / nthreads), hi = int(int64_t(n) * (t + 1) / nthreads);
    std::vector<uint32_t> cps;
    std::vector<std::vector<uint32_t>> words;
    std::vector<int32_t> sent;
    std::vector<int32_t>& out = part[size_t(t)];
    for (int i = lo; i < hi; ++i) {
      utf8_decode(texts[i], &cps);
      normalize_and_split(*v, cps, &words);
      sent.clear();
      for (const auto& w : words) {
        wordpiece(*v, w, &sent);
        if (int(sent.size()) >= max_len - 2) break;
      }
      if (int(sent.size()) > max_len - 2) sent.resize(size_t(max_len - 2));
      out.push_back(v->cls);
      out.insert(out.end(), sent.begin(), sent.end());
      out.push_back(v->sep);
      lens[size_t(i)] = int32_t(sent.size()) + 2;
    }
  };
  if (nthreads == 1) {
    work(0);
  } else {
    std::vector<std::thread> pool;
    for (int t = 0; t < nthreads; ++t) pool.emplace_back(work, t);
    for (auto& th : pool) th.join();
  }
  int64_t pos = 0;
  cu_seqlens[0] = 0;
  for (int i = 0; i < n; ++i) {
    pos += lens[size_t(i)];
    if (pos > INT32_MAX) return bbh::internal_fail(BBH_ERR_CAPACITY, "bbh_tokenize: more than 2^31 tokens");
    cu_seqlens[i + 1] = int32_t(pos);
  }
  *total = pos;
  if (pos > ids_cap)
    return bbh::internal_fail(BBH_ERR_CAPACITY, "bbh_tokenize: ids needs " + std::to_string(pos) + " entries, has " +
                                                    std::to_string(ids_cap));
  int64_t at = 0;
  for (const auto& pbuf : part) {
    std::memcpy(ids + at, pbuf.data(), pbuf.size() * sizeof(int32_t));
    at += int64_t(pbuf.size());
  }
  return BBH_OK;
}

}  // extern "C"

// text.cu -- streaming detokenization, host side (no device code).
//
// Restates the reference's incremental text decoder (cmd/monolith/monolith.go,
// "M:line"): incrementalText.Push (M:7703-7733), its HF ByteLevel branch
// pushHF (M:7737-7780), Transformers' cleanup cascade clean (M:7672-7701) and
// the Mistral byte-fallback PushToken (M:2132-2161).  The engine feeds each
// sampled token's piece (the tokenizer's bytes for that id) and gets back the
// text that can be shown so far, so concatenated deltas equal the whole-string
// decode even when a token ends inside a UTF-8 sequence or a cleanup pattern.
// Tokenization itself (the pieces table) stays with the caller.
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/srstep.h"
#include "srstep_internal.h"

namespace {

const char kReplacement[] = "\xEF\xBF\xBD";  // U+FFFD

// Width of the UTF-8 sequence a lead byte announces (Go's utf8 "first" table),
// 1 for ASCII and for bytes that can never start a sequence.
int lead_size(uint8_t b) {
  if (b < 0x80) return 1;
  if (b >= 0xC2 && b <= 0xDF) return 2;
  if (b >= 0xE0 && b <= 0xEF) return 3;
  if (b >= 0xF0 && b <= 0xF4) return 4;
  return 1;
}
bool lead_invalid(uint8_t b) { return b >= 0x80 && lead_size(b) == 1; }
// Accepted range of the second byte (Go's acceptRanges).
void second_range(uint8_t b, uint8_t* lo, uint8_t* hi) {
  *lo = 0x80;
  *hi = 0xBF;
  if (b == 0xE0) *lo = 0xA0;
  else if (b == 0xED) *hi = 0x9F;
  else if (b == 0xF0) *lo = 0x90;
  else if (b == 0xF4) *hi = 0x8F;
}

// utf8.FullRune: p begins with a complete rune, or with bytes that can only
// decode as a width-1 error.
bool full_rune(const uint8_t* p, size_t n) {
  if (n == 0) return false;
  const int sz = lead_size(p[0]);
  if ((int)n >= sz) return true;
  uint8_t lo, hi;
  second_range(p[0], &lo, &hi);
  if (n > 1 && (p[1] < lo || hi < p[1])) return true;
  if (n > 2 && (p[2] < 0x80 || 0xBF < p[2])) return true;
  return false;
}

// utf8.DecodeRune's width and validity (RuneError with width 1 when invalid).
int decode_width(const uint8_t* p, size_t n, bool* valid) {
  *valid = false;
  const uint8_t b = p[0];
  if (b < 0x80) {
    *valid = true;
    return 1;
  }
  if (lead_invalid(b)) return 1;
  const int sz = lead_size(b);
  if ((int)n < sz) return 1;
  uint8_t lo, hi;
  second_range(b, &lo, &hi);
  if (p[1] < lo || hi < p[1]) return 1;
  for (int k = 2; k < sz; k++)
    if (p[k] < 0x80 || 0xBF < p[k]) return 1;
  *valid = true;
  return sz;
}

bool valid_utf8(const std::string& s) {
  const uint8_t* p = (const uint8_t*)s.data();
  for (size_t i = 0; i < s.size();) {
    bool ok;
    const int w = decode_width(p + i, s.size() - i, &ok);
    if (!ok) return false;
    i += w;
  }
  return true;
}

// Transformers' ordered cleanup replacements (hfCleanup, M:7672-7676).
const char* const kCleanup[10][2] = {{" .", "."},     {" ?", "?"},     {" !", "!"},     {" ,", ","},
                                     {" ' ", "'"},    {" n't", "n't"}, {" 'm", "'m"},   {" 's", "'s"},
                                     {" 've", "'ve"}, {" 're", "'re"}};

}  // namespace

struct sr_text_decoder {
  bool hf = false, cleanup = false, mistral = false, leading = false;
  bool invalid = false;         // incrementalText.invalid
  std::string pending;          // incrementalText.pending
  std::string held[10];         // incrementalText.held
  std::vector<uint8_t> fallback;  // Mistral byte-fallback ids (hfTokenizer.fallback)
  std::string ready;            // decoded text not yet handed to the caller

  // incrementalText.clean (M:7678-7701): each stage keeps back only a possible
  // prefix of its pattern.
  std::string clean(std::string text, bool final) {
    for (int i = 0; i < 10; i++) {
      const std::string pat = kCleanup[i][0], rep = kCleanup[i][1];
      text = held[i] + text;
      held[i].clear();
      std::string out;
      size_t at;
      while ((at = text.find(pat)) != std::string::npos) {
        out.append(text, 0, at);
        out += rep;
        text.erase(0, at + pat.size());
      }
      size_t keep = 0;
      if (!final)
        for (size_t n = 1; n < pat.size() && n <= text.size(); n++)
          if (text.compare(text.size() - n, n, pat, 0, n) == 0) keep = n;
      out.append(text, 0, text.size() - keep);
      held[i] = text.substr(text.size() - keep);
      text = out;
    }
    return text;
  }

  // Push's plain branch (M:7712-7733): strings.ToValidUTF8 across pieces, one
  // replacement per run of invalid bytes.
  std::string push_plain(const std::string& piece, bool final) {
    std::string data = pending + piece;
    pending.clear();
    std::string out;
    const uint8_t* p = (const uint8_t*)data.data();
    for (size_t i = 0; i < data.size();) {
      if (!final && !full_rune(p + i, data.size() - i)) {
        pending.assign(data, i, std::string::npos);
        break;
      }
      bool ok;
      const int w = decode_width(p + i, data.size() - i, &ok);
      if (!ok) {
        if (!invalid) out += kReplacement;
        invalid = true;
      } else {
        out.append(data, i, w);
        invalid = false;
      }
      i += w;
    }
    return out;
  }

  // pushHF (M:7737-7780): the ByteLevel decoder's lossy UTF-8 (one replacement
  // per maximal invalid subpart), holding back an incomplete valid prefix.
  std::string push_hf(const std::string& piece, bool final) {
    std::string data = pending + piece;
    pending.clear();
    std::string out;
    const uint8_t* p = (const uint8_t*)data.data();
    const size_t len = data.size();
    for (size_t pos = 0; pos < len;) {
      const uint8_t b = p[pos];
      if (b < 0x80) {
        out += (char)b;
        pos++;
        continue;
      }
      const int need = lead_invalid(b) ? 1 : lead_size(b);
      int n = 1;
      while (n < need && pos + n < len) {
        const uint8_t c = p[pos + n];
        if (c < 0x80 || c > 0xBF ||
            (n == 1 && ((b == 0xE0 && c < 0xA0) || (b == 0xED && c >= 0xA0) || (b == 0xF0 && c < 0x90) ||
                        (b == 0xF4 && c >= 0x90))))
          break;
        n++;
      }
      if (need > 1 && n == need) {
        out.append(data, pos, n);
        pos += n;
        continue;
      }
      if (need > 1 && pos + n == len && n < need && !final) {
        pending.assign(data, pos, std::string::npos);
        break;
      }
      out += kReplacement;
      pos += n;
    }
    return out;
  }

  // incrementalText.Push (M:7703-7711).
  std::string push(const std::string& piece, bool final) {
    if (hf) {
      std::string text = push_hf(piece, final);
      return cleanup ? clean(text, final) : text;
    }
    return push_plain(piece, final);
  }

  // PushToken (M:2132-2161): a run of byte-fallback tokens decodes atomically
  // (one replacement per byte if the run is not valid UTF-8); the first
  // non-empty text loses one leading space.
  std::string push_token(int32_t id, const std::string& piece, bool final) {
    if (!mistral) return push(piece, final);
    std::string out;
    auto flush = [&] {
      if (valid_utf8(pending)) out += pending;
      else
        for (size_t k = 0; k < pending.size(); k++) out += kReplacement;
      pending.clear();
    };
    if (id >= 0 && (size_t)id < fallback.size() && fallback[id]) pending += piece;
    else if (!piece.empty()) {
      flush();
      out += piece;
    }
    if (final) flush();
    if (leading && !out.empty()) {
      if (out[0] == ' ') out.erase(0, 1);
      leading = false;
    }
    return out;
  }

  // Hand over as much of `ready` as fits in cap bytes, ending on a character
  // boundary; the rest waits for the next call.
  void take(char* dst, int64_t cap, int64_t* n_out, int64_t* queued) {
    size_t n = std::min<size_t>(ready.size(), cap > 0 ? (size_t)cap : 0);
    while (n > 0 && n < ready.size() && ((uint8_t)ready[n] & 0xC0) == 0x80) n--;
    if (n) memcpy(dst, ready.data(), n);
    ready.erase(0, n);
    *n_out = (int64_t)n;
    if (queued) *queued = (int64_t)ready.size();
  }
};

extern "C" int sr_text_decoder_create(int32_t flags, const uint8_t* fallback, int32_t vocab, sr_text_decoder** out) {
  if (!out) return sr_fail(SR_EINVAL, "null argument");
  *out = nullptr;
  if (flags & ~(SR_TEXT_HF | SR_TEXT_CLEANUP | SR_TEXT_MISTRAL)) return sr_fail(SR_EINVAL, "unknown text flags");
  if ((flags & SR_TEXT_CLEANUP) && !(flags & SR_TEXT_HF))
    return sr_fail(SR_EINVAL, "cleanup applies to HF tokenizers only");  // cleanup: ok && h.cleanup (M:7663)
  if ((flags & SR_TEXT_MISTRAL) && (vocab < 0 || (vocab > 0 && !fallback)))
    return sr_fail(SR_EINVAL, "the Mistral decoder needs the byte-fallback flags of the vocabulary");
  sr_text_decoder* d = new sr_text_decoder();
  d->hf = (flags & SR_TEXT_HF) != 0;
  d->cleanup = (flags & SR_TEXT_CLEANUP) != 0;
  d->mistral = d->leading = (flags & SR_TEXT_MISTRAL) != 0;
  if (d->mistral && vocab > 0) d->fallback.assign(fallback, fallback + vocab);
  *out = d;
  return SR_OK;
}

extern "C" int sr_text_decoder_destroy(sr_text_decoder* d) {
  if (!d) return sr_fail(SR_EINVAL, "null decoder");
  delete d;
  return SR_OK;
}

extern "C" int sr_text_decoder_push(sr_text_decoder* d, const uint8_t* bytes, int64_t n, int32_t final, char* out,
                                    int64_t cap, int64_t* n_out, int64_t* queued) {
  if (!d || !n_out || (n > 0 && !bytes) || n < 0 || (cap > 0 && !out)) return sr_fail(SR_EINVAL, "invalid argument");
  d->ready += d->push(std::string((const char*)bytes, n > 0 ? (size_t)n : 0), final != 0);
  d->take(out, cap, n_out, queued);
  return SR_OK;
}

extern "C" int sr_text_decoder_push_token(sr_text_decoder* d, int32_t id, const uint8_t* piece, int64_t n,
                                          int32_t final, char* out, int64_t cap, int64_t* n_out, int64_t* queued) {
  if (!d || !n_out || (n > 0 && !piece) || n < 0 || (cap > 0 && !out)) return sr_fail(SR_EINVAL, "invalid argument");
  d->ready += d->push_token(id, std::string((const char*)piece, n > 0 ? (size_t)n : 0), final != 0);
  d->take(out, cap, n_out, queued);
  return SR_OK;
}

// segmenter.cpp -- bounded, tokenizer-aware splitting of long source text.
//
// Restates segment_text (crates/marian-core/src/segmenter.rs:122-197) and its
// helpers: the input is split into ordered, lossless (content, separator)
// byte ranges whose content fits a source-piece limit, preferring sentence
// and line boundaries, then clause punctuation, commas, whitespace, and
// finally the largest prefix of whole UTF-8 scalars.  The caller supplies
// the exact piece counter (its tokenizer); separators are preserved verbatim
// and never translated.  Work done through the counter is bounded the way
// the reference bounds it (segmenter.rs:13-22).
//
// The reference operates on a Rust &str; here the bytes are validated as
// UTF-8 first (an invalid sequence is an input error), after which every
// helper below steps by whole scalars as the reference's char iteration does.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <utility>
#include <vector>

#include "marian_cuda.h"

namespace {

constexpr size_t kMaxInputBytes = 4u * 1024 * 1024;     // segmenter.rs:14
constexpr size_t kMaxSegments = 4096;                    // segmenter.rs:16
constexpr size_t kMaxEncodingCalls = 32768;              // segmenter.rs:18
constexpr size_t kMaxEncodingBytes = 64u * 1024 * 1024;  // segmenter.rs:20
constexpr size_t kMaxCountedPieces = 8u * 1024 * 1024;   // segmenter.rs:22

struct Range {
  size_t start, end;
};

struct Unit {
  Range content, separator;
};

struct BreakPoint {
  size_t content_end, next_start;
  int priority;
};

struct Segment {
  Range content, separator;
  size_t pieces;
};

// A failure carried up to the C ABI (segmenter.rs:48-110).
struct Failure {
  int32_t kind = MC_SEGMENT_OK;
  uint64_t start = 0, end = 0, pieces = 0, maximum = 0;
  std::string message;
};

std::string format(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return buf;
}

// ---- UTF-8 scalars -------------------------------------------------------------
class Text {
 public:
  Text(const char* p, size_t n) : p_(reinterpret_cast<const unsigned char*>(p)), n_(n) {}
  size_t size() const { return n_; }
  unsigned char byte(size_t i) const { return p_[i]; }
  const char* data() const { return reinterpret_cast<const char*>(p_); }

  bool is_char_boundary(size_t i) const { return i == 0 || i >= n_ || (p_[i] & 0xC0) != 0x80; }

  // The scalar starting at i (i < size, on a boundary) and the index after it.
  std::pair<uint32_t, size_t> next(size_t i) const {
    const unsigned char b = p_[i];
    if (b < 0x80) return {b, i + 1};
    if (b < 0xE0) return {((b & 0x1Fu) << 6) | (p_[i + 1] & 0x3Fu), i + 2};
    if (b < 0xF0) return {((b & 0x0Fu) << 12) | ((p_[i + 1] & 0x3Fu) << 6) | (p_[i + 2] & 0x3Fu), i + 3};
    return {((b & 0x07u) << 18) | ((p_[i + 1] & 0x3Fu) << 12) | ((p_[i + 2] & 0x3Fu) << 6) |
                (p_[i + 3] & 0x3Fu),
            i + 4};
  }

  // The scalar ending at end (end > 0, on a boundary): its start and value.
  std::pair<size_t, uint32_t> previous(size_t end) const {
    size_t s = end - 1;
    while (s > 0 && (p_[s] & 0xC0) == 0x80) --s;
    return {s, next(s).first};
  }

  // Strict UTF-8 (shortest forms, no surrogates, at most U+10FFFF).
  bool valid() const {
    size_t i = 0;
    while (i < n_) {
      const unsigned char b = p_[i];
      size_t len;
      uint32_t cp, min;
      if (b < 0x80) {
        ++i;
        continue;
      } else if ((b & 0xE0) == 0xC0) {
        len = 2, cp = b & 0x1F, min = 0x80;
      } else if ((b & 0xF0) == 0xE0) {
        len = 3, cp = b & 0x0F, min = 0x800;
      } else if ((b & 0xF8) == 0xF0) {
        len = 4, cp = b & 0x07, min = 0x10000;
      } else {
        return false;
      }
      if (i + len > n_) return false;
      for (size_t k = 1; k < len; ++k) {
        if ((p_[i + k] & 0xC0) != 0x80) return false;
        cp = (cp << 6) | (p_[i + k] & 0x3F);
      }
      if (cp < min || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
      i += len;
    }
    return true;
  }

 private:
  const unsigned char* p_;
  size_t n_;
};

// Unicode White_Space, the set Rust's char::is_whitespace tests.
bool is_whitespace(uint32_t c) {
  return (c >= 0x09 && c <= 0x0D) || c == 0x20 || c == 0x85 || c == 0xA0 || c == 0x1680 ||
         (c >= 0x2000 && c <= 0x200A) || c == 0x2028 || c == 0x2029 || c == 0x202F || c == 0x205F ||
         c == 0x3000;
}

bool is_ascii_digit(uint32_t c) { return c >= '0' && c <= '9'; }
bool is_ascii_alpha(uint32_t c) { return (c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z'); }
bool is_ascii_upper(uint32_t c) { return c >= 'A' && c <= 'Z'; }
bool is_ascii_lower(uint32_t c) { return c >= 'a' && c <= 'z'; }

// segmenter.rs:594-599
bool is_terminator(uint32_t c) {
  return c == '.' || c == '!' || c == '?' || c == 0x3002 || c == 0xFF01 || c == 0xFF1F || c == 0x2026;
}

// segmenter.rs:550-577
bool is_closing_mark(uint32_t c) {
  switch (c) {
    case '"': case '\'': case 0x2019: case 0x201D: case 0x00BB: case ')': case ']': case '}':
    case 0x3009: case 0x300B: case 0x300D: case 0x300F: case 0x3011: case 0x3015: case 0x3017:
    case 0x3019: case 0x301B:
      return true;
    default:
      return false;
  }
}

size_t consume_terminators(const Text& t, size_t i, size_t end) {
  while (i < end) {
    auto [c, n] = t.next(i);
    if (!is_terminator(c)) break;
    i = n;
  }
  return i;
}

size_t consume_closing_marks(const Text& t, size_t i, size_t end) {
  while (i < end) {
    auto [c, n] = t.next(i);
    if (!is_closing_mark(c)) break;
    i = n;
  }
  return i;
}

size_t consume_whitespace(const Text& t, size_t i, size_t end) {
  while (i < end) {
    auto [c, n] = t.next(i);
    if (!is_whitespace(c)) break;
    i = n;
  }
  return i;
}

size_t trim_trailing_whitespace(const Text& t, size_t end) {
  while (end > 0) {
    auto [s, c] = t.previous(end);
    if (!is_whitespace(c)) break;
    end = s;
  }
  return end;
}

bool boundary_follows(const Text& t, size_t i, size_t end) {
  return i == end || (i < end && is_whitespace(t.next(i).first));
}

// segmenter.rs:643-661
const char* const kTitleAbbreviations[] = {"capt.", "col.", "dr.",  "gen.", "gov.", "lt.",  "mr.", "mrs.",
                                           "ms.",   "prof.", "rep.", "rev.", "sen.", "sgt.", "sr.", "st."};
const char* const kNonTerminalAbbreviations[] = {"e.g.", "i.e.", "fig.", "no.",  "vs.",  "jan.",
                                                 "feb.", "mar.", "apr.", "jun.", "jul.", "aug.",
                                                 "sep.", "sept.", "oct.", "nov.", "dec."};
const char* const kCommonAbbreviations[] = {"approx.", "co.",  "corp.", "dept.", "ed.", "eds.", "est.",
                                            "etc.",    "inc.", "ltd.",  "misc.", "p.",  "pp.",  "vol."};

template <size_t N>
bool listed(const char* const (&table)[N], const std::string& token) {
  for (const char* entry : table)
    if (token == entry) return true;
  return false;
}

// segmenter.rs:663-670: dot-separated single ASCII letters ("u.s.", "j.").
bool is_initial_or_acronym(const std::string& token) {
  size_t end = token.size();
  while (end > 0 && token[end - 1] == '.') --end;
  const std::string core = token.substr(0, end);
  size_t components = 0, start = 0;
  for (;;) {
    const size_t dot = core.find('.', start);
    const size_t stop = dot == std::string::npos ? core.size() : dot;
    if (stop - start != 1 || !is_ascii_alpha(static_cast<unsigned char>(core[start]))) return false;
    ++components;
    if (dot == std::string::npos) break;
    start = dot + 1;
  }
  return components <= 8;
}

// segmenter.rs:601-641: whether the '.' at `index` (whose terminators and
// closing marks end at quoted_end) ends a sentence.
bool period_can_end_sentence(const Text& t, size_t index, size_t quoted_end) {
  bool has_prev = index > 0, has_next = index + 1 < t.size();
  const uint32_t prev = has_prev ? t.previous(index).second : 0;
  const uint32_t next = has_next ? t.next(index + 1).first : 0;
  if (has_prev && is_ascii_digit(prev) && has_next && is_ascii_digit(next)) return false;

  size_t token_start = 0;
  for (size_t e = index; e > 0;) {
    auto [s, c] = t.previous(e);
    if (is_whitespace(c) || c == '(' || c == '[' || c == '{' || c == '"' || c == 0x201C) {
      token_start = e;
      break;
    }
    e = s;
  }
  std::string token;
  for (size_t i = token_start; i <= index; ++i) {
    unsigned char b = t.byte(i);
    if (b >= 'A' && b <= 'Z') b = static_cast<unsigned char>(b - 'A' + 'a');
    if ((b >= 'a' && b <= 'z') || (b >= '0' && b <= '9') || b == '.') token.push_back(static_cast<char>(b));
  }

  const size_t f = consume_whitespace(t, quoted_end, t.size());
  const bool has_following = f < t.size();
  const uint32_t following = has_following ? t.next(f).first : 0;
  if (listed(kTitleAbbreviations, token) && has_following) return false;
  if (listed(kNonTerminalAbbreviations, token) && has_following) return false;
  if (listed(kCommonAbbreviations, token) && has_following &&
      (is_ascii_lower(following) || is_ascii_digit(following)))
    return false;
  if (is_initial_or_acronym(token) && has_following && is_ascii_upper(following)) return false;
  return true;
}

// segmenter.rs:267-320: sentence and line units of text[0, content_end).
std::vector<Unit> sentence_units(const Text& t, size_t content_end) {
  std::vector<Unit> units;
  size_t cursor = 0, index = 0;
  while (index < content_end) {
    auto [c, next] = t.next(index);
    if (is_terminator(c)) {
      const size_t punct_end = consume_terminators(t, index, content_end);
      const size_t quoted_end = consume_closing_marks(t, punct_end, content_end);
      if (boundary_follows(t, quoted_end, content_end) &&
          (c != '.' || period_can_end_sentence(t, index, quoted_end))) {
        const size_t sep_end = consume_whitespace(t, quoted_end, content_end);
        units.push_back({{cursor, quoted_end}, {quoted_end, sep_end}});
        cursor = sep_end;
        index = sep_end;
        continue;
      }
      index = punct_end > next ? punct_end : next;
      continue;
    }
    if (is_whitespace(c)) {
      const size_t ws_end = consume_whitespace(t, index, content_end);
      bool line_break = false;
      for (size_t i = index; i < ws_end; ++i)
        if (t.byte(i) == '\n' || t.byte(i) == '\r') line_break = true;
      if (line_break) {
        units.push_back({{cursor, index}, {index, ws_end}});
        cursor = ws_end;
      }
      index = ws_end;
      continue;
    }
    index = next;
  }
  if (cursor < content_end) {
    units.push_back({{cursor, content_end}, {content_end, t.size()}});
  } else if (!units.empty()) {
    units.back().separator.end = t.size();
  }
  return units;
}

// segmenter.rs:672-679
bool is_dash_boundary(const Text& t, size_t index, Range r) {
  const bool repeated = index + 1 < r.end && t.byte(index + 1) == '-';
  const bool before_space = index == r.start || is_whitespace(t.previous(index).second);
  const size_t after = index + 1;
  const bool after_space = after >= r.end || is_whitespace(t.next(after).first);
  return repeated || before_space || after_space;
}

// segmenter.rs:475-516: candidate breaks inside an oversize unit, priority
// 0 (clause punctuation and dashes), 1 (commas) or 2 (whitespace).
std::vector<BreakPoint> fallback_break_points(const Text& t, Range r) {
  std::vector<BreakPoint> points;
  size_t index = r.start;
  while (index < r.end) {
    auto [c, next] = t.next(index);
    if (is_whitespace(c)) {
      const size_t end = consume_whitespace(t, index, r.end);
      points.push_back({index, end, 2});
      index = end;
      continue;
    }
    int priority = -1;
    if (c == ';' || c == 0xFF1B || c == ':' || c == 0xFF1A || c == '/' || c == 0x2013 || c == 0x2014)
      priority = 0;
    else if (c == ',' || c == 0xFF0C)
      priority = 1;
    else if (c == '-' && is_dash_boundary(t, index, r))
      priority = 0;
    if (priority >= 0) {
      size_t punct_end = next;
      if (c == '-')
        while (punct_end < r.end && t.byte(punct_end) == '-') ++punct_end;
      const size_t sep_end = consume_whitespace(t, punct_end, r.end);
      points.push_back({punct_end, sep_end, priority});
      index = punct_end;
      continue;
    }
    index = next;
  }
  return points;
}

// segmenter.rs:186-265: memoized, bounded calls of the caller's counter.
class PieceCounter {
 public:
  PieceCounter(const Text& t, mc_piece_count_fn fn, void* ctx) : t_(t), fn_(fn), ctx_(ctx) {}

  bool count(Range r, size_t* out, Failure* f) {
    auto it = cache_.find({r.start, r.end});
    if (it != cache_.end()) {
      *out = it->second;
      return true;
    }
    if (++calls_ > kMaxEncodingCalls) return limit(f, "tokenizer calls", kMaxEncodingCalls);
    bytes_ += r.end - r.start;
    if (bytes_ > kMaxEncodingBytes) return limit(f, "encoded bytes", kMaxEncodingBytes);
    uint64_t pieces = 0;
    char msg[256] = {0};
    const int32_t rc = fn_(ctx_, t_.data() + r.start, r.end - r.start, &pieces, msg, sizeof(msg));
    if (rc != 0) {
      msg[sizeof(msg) - 1] = 0;
      f->kind = MC_SEGMENT_ENCODING;
      f->start = r.start;
      f->end = r.end;
      f->message = format("source tokenizer failed for byte range %zu..%zu: %s", r.start, r.end, msg);
      return false;
    }
    pieces_ += pieces;
    if (pieces_ > kMaxCountedPieces) return limit(f, "counted pieces", kMaxCountedPieces);
    cache_[{r.start, r.end}] = static_cast<size_t>(pieces);
    *out = static_cast<size_t>(pieces);
    return true;
  }

 private:
  static bool limit(Failure* f, const char* resource, size_t maximum) {
    f->kind = MC_SEGMENT_ENCODING_WORK_LIMIT;
    f->maximum = maximum;
    f->message = format("source segmentation exceeded %s safety limit %zu", resource, maximum);
    return false;
  }

  const Text& t_;
  mc_piece_count_fn fn_;
  void* ctx_;
  std::map<std::pair<size_t, size_t>, size_t> cache_;
  size_t calls_ = 0, bytes_ = 0, pieces_ = 0;
};

bool push_segment(std::vector<Segment>& result, const Segment& s, Failure* f) {
  if (result.size() >= kMaxSegments) {
    f->kind = MC_SEGMENT_TOO_MANY_SEGMENTS;
    f->maximum = kMaxSegments;
    f->message = format("source requires more than %zu segments", kMaxSegments);
    return false;
  }
  result.push_back(s);
  return true;
}

size_t floor_char_boundary(const Text& t, size_t index, size_t minimum) {
  while (index > minimum && !t.is_char_boundary(index)) --index;
  return index;
}

size_t previous_char_boundary(const Text& t, size_t index, size_t minimum) {
  if (index <= minimum) return minimum;
  size_t previous = index - 1;
  while (previous > minimum && !t.is_char_boundary(previous)) --previous;
  return previous;
}

// segmenter.rs:392-432: the rightmost break of one priority whose prefix
// fits, by binary search over the candidates in text order.
bool rightmost_fitting_break(const std::vector<BreakPoint>& points, int priority, size_t start,
                             size_t end, size_t max_pieces, PieceCounter& counter, bool* found,
                             BreakPoint* best, size_t* best_pieces, Failure* f) {
  std::vector<BreakPoint> candidates;
  for (const BreakPoint& p : points)
    if (p.priority == priority && p.content_end > start && p.next_start > start && p.next_start < end)
      candidates.push_back(p);
  *found = false;
  size_t low = 0, high = candidates.size();
  while (low < high) {
    const size_t middle = low + (high - low) / 2;
    size_t pieces = 0;
    if (!counter.count({start, candidates[middle].content_end}, &pieces, f)) return false;
    if (pieces <= max_pieces) {
      *found = true;
      *best = candidates[middle];
      *best_pieces = pieces;
      low = middle + 1;
    } else {
      high = middle;
    }
  }
  return true;
}

// segmenter.rs:434-473: the longest prefix of whole scalars that fits.
bool largest_fitting_scalar_prefix(const Text& t, size_t start, size_t end, size_t max_pieces,
                                   PieceCounter& counter, size_t* out_end, size_t* out_pieces,
                                   Failure* f) {
  const size_t first_end = t.next(start).second;
  size_t first_pieces = 0;
  if (!counter.count({start, first_end}, &first_pieces, f)) return false;
  if (first_pieces > max_pieces) {
    f->kind = MC_SEGMENT_UNSPLITABLE_SCALAR;
    f->start = start;
    f->end = first_end;
    f->pieces = first_pieces;
    f->maximum = max_pieces;
    f->message = format("UTF-8 scalar at byte range %zu..%zu encodes to %zu pieces; maximum is %zu", start,
                        first_end, first_pieces, max_pieces);
    return false;
  }
  size_t low = first_end, high = end;
  size_t best_end = first_end, best_pieces = first_pieces;
  while (low < high) {
    const size_t raw_middle = low + (high - low + 1) / 2;
    const size_t middle = floor_char_boundary(t, raw_middle, start);
    if (middle <= best_end) break;
    size_t pieces = 0;
    if (!counter.count({start, middle}, &pieces, f)) return false;
    if (pieces <= max_pieces) {
      best_end = middle;
      best_pieces = pieces;
      low = middle;
    } else {
      high = previous_char_boundary(t, middle, start);
    }
  }
  *out_end = best_end;
  *out_pieces = best_pieces;
  return true;
}

// segmenter.rs:322-390
bool split_oversize_unit(const Text& t, const Unit& unit, size_t max_pieces, PieceCounter& counter,
                         std::vector<Segment>& result, Failure* f) {
  const std::vector<BreakPoint> points = fallback_break_points(t, unit.content);
  size_t start = unit.content.start;
  while (start < unit.content.end) {
    size_t remaining = 0;
    if (!counter.count({start, unit.content.end}, &remaining, f)) return false;
    if (remaining <= max_pieces)
      return push_segment(result, {{start, unit.content.end}, unit.separator, remaining}, f);
    bool found = false;
    BreakPoint point{};
    size_t pieces = 0;
    for (int priority = 0; priority <= 2 && !found; ++priority)
      if (!rightmost_fitting_break(points, priority, start, unit.content.end, max_pieces, counter, &found,
                                   &point, &pieces, f))
        return false;
    size_t content_end, next_start;
    if (found) {
      content_end = point.content_end;
      next_start = point.next_start;
    } else {
      size_t end = 0;
      if (!largest_fitting_scalar_prefix(t, start, unit.content.end, max_pieces, counter, &end, &pieces, f))
        return false;
      content_end = next_start = end;
    }
    if (!push_segment(result, {{start, content_end}, {content_end, next_start}, pieces}, f)) return false;
    start = next_start;
  }
  if (unit.separator.start < unit.separator.end && !result.empty())
    result.back().separator.end = unit.separator.end;
  return true;
}

// segmenter.rs:122-175
bool segment_text(const Text& t, size_t max_pieces, mc_piece_count_fn fn, void* ctx,
                  std::vector<Segment>& result, Failure* f) {
  if (max_pieces == 0) {
    f->kind = MC_SEGMENT_ZERO_PIECE_LIMIT;
    f->message = "source piece limit must be non-zero";
    return false;
  }
  if (t.size() > kMaxInputBytes) {
    f->kind = MC_SEGMENT_INPUT_TOO_LARGE;
    f->end = t.size();
    f->maximum = kMaxInputBytes;
    f->message = format("source contains %zu bytes; segmenter maximum is %zu", t.size(), kMaxInputBytes);
    return false;
  }
  if (!t.valid()) {
    f->kind = MC_SEGMENT_INVALID_UTF8;
    f->message = "source text is not valid UTF-8";
    return false;
  }
  const size_t content_end = trim_trailing_whitespace(t, t.size());
  PieceCounter counter(t, fn, ctx);
  size_t whole = 0;
  if (!counter.count({0, content_end}, &whole, f)) return false;
  const std::vector<Unit> units = sentence_units(t, content_end);
  if (whole <= max_pieces && units.size() <= 1) {
    result.push_back({{0, content_end}, {content_end, t.size()}, whole});
    return true;
  }
  for (const Unit& unit : units) {
    size_t pieces = 0;
    if (!counter.count(unit.content, &pieces, f)) return false;
    if (pieces <= max_pieces) {
      if (!push_segment(result, {unit.content, unit.separator, pieces}, f)) return false;
    } else if (!split_oversize_unit(t, unit, max_pieces, counter, result, f)) {
      return false;
    }
  }
  return true;
}

void set_error(mc_segment_error* e, const Failure& f) {
  if (!e) return;
  e->kind = f.kind;
  e->start = f.start;
  e->end = f.end;
  e->pieces = f.pieces;
  e->maximum = f.maximum;
  std::snprintf(e->message, sizeof(e->message), "%s", f.message.c_str());
}

}  // namespace

extern "C" mc_status mc_segment_text(const char* text, size_t len, uint64_t max_pieces,
                                     mc_piece_count_fn count_pieces, void* ctx,
                                     mc_text_segment* segments, size_t capacity, size_t* n_segments,
                                     mc_segment_error* error) {
  Failure f;
  if (n_segments) *n_segments = 0;
  if ((!text && len) || !count_pieces || !n_segments) {
    f.kind = MC_SEGMENT_INVALID_ARGUMENT;
    f.message = "text, count_pieces and n_segments are required";
    set_error(error, f);
    return MC_INVALID_INPUT;
  }
  const Text t(text ? text : "", len);
  std::vector<Segment> result;
  if (!segment_text(t, static_cast<size_t>(max_pieces), count_pieces, ctx, result, &f)) {
    set_error(error, f);
    return MC_INVALID_INPUT;
  }
  *n_segments = result.size();
  if (result.size() > capacity || (!segments && !result.empty())) {
    f.kind = MC_SEGMENT_INVALID_ARGUMENT;
    f.message = format("%zu segments do not fit the capacity %zu", result.size(), capacity);
    set_error(error, f);
    return MC_INVALID_INPUT;
  }
  for (size_t i = 0; i < result.size(); ++i) {
    segments[i].content_start = result[i].content.start;
    segments[i].content_end = result[i].content.end;
    segments[i].separator_start = result[i].separator.start;
    segments[i].separator_end = result[i].separator.end;
    segments[i].source_pieces = result[i].pieces;
  }
  set_error(error, f);  // kind MC_SEGMENT_OK, empty message
  return MC_OK;
}

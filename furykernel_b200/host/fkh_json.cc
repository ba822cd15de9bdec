// Just enough JSON for selections (src/FuryKernel/Json.hs): writing is
// deterministic -- keys in the order given, two-space indentation, a final
// newline -- and reading takes RFC 8259 JSON except that numbers must be
// integers (here: within int64) and an object's keys must be unique. A
// reading error names what is wrong and the character (code point) where.
#include <cerrno>
#include <cstdio>
#include <cstdlib>
#include <tuple>

#include "fkh_select.h"

namespace fkh {

namespace {

void put_utf8(std::string& out, uint32_t c) {
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

std::string quoted(const std::string& s) {
  std::string out = "\"";
  for (unsigned char c : s) {
    switch (c) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      default:
        if (c < 0x20) {
          char buf[8];
          std::snprintf(buf, sizeof buf, "\\u%04x", c);
          out += buf;
        } else {
          out += (char)c;
        }
    }
  }
  return out + "\"";
}

void render(const Json& j, int depth, std::string& out) {
  const std::string pad((size_t)2 * (depth + 1), ' '), close((size_t)2 * depth, ' ');
  switch (j.kind) {
    case Json::Null: out += "null"; break;
    case Json::Bool: out += j.b ? "true" : "false"; break;
    case Json::Int: out += std::to_string(j.i); break;
    case Json::String: out += quoted(j.s); break;
    case Json::Array:
      if (j.items.empty()) {
        out += "[]";
        break;
      }
      out += "[\n";
      for (size_t k = 0; k < j.items.size(); ++k) {
        out += (k ? ",\n" : "") + pad;
        render(j.items[k], depth + 1, out);
      }
      out += "\n" + close + "]";
      break;
    case Json::Object:
      if (j.members.empty()) {
        out += "{}";
        break;
      }
      out += "{\n";
      for (size_t k = 0; k < j.members.size(); ++k) {
        out += (k ? ",\n" : "") + pad + quoted(j.members[k].first) + ": ";
        render(j.members[k].second, depth + 1, out);
      }
      out += "\n" + close + "}";
      break;
  }
}

struct Reader {
  const std::string& in;
  size_t at = 0;

  // The character offset of a byte offset: code points before it.
  size_t chars(size_t byte) const {
    size_t n = 0;
    for (size_t i = 0; i < byte && i < in.size(); ++i)
      if (((unsigned char)in[i] & 0xC0) != 0x80) ++n;
    return n;
  }
  [[noreturn]] void fail(size_t where, const std::string& what) const {
    throw Refusal(what + " at character " + std::to_string(chars(where)) + ".");
  }
  void skip() {
    while (at < in.size() && (in[at] == ' ' || in[at] == '\t' || in[at] == '\n' || in[at] == '\r')) ++at;
  }
  bool starts(const char* w) const { return in.compare(at, std::char_traits<char>::length(w), w) == 0; }

  Json value() {
    if (at >= in.size()) fail(at, "No JSON value");
    const char c = in[at];
    if (c == '{') {
      ++at;
      skip();
      return object();
    }
    if (c == '[') {
      ++at;
      skip();
      return array();
    }
    if (c == '"') {
      ++at;
      Json j;
      j.kind = Json::String;
      j.s = string_body();
      skip();
      return j;
    }
    if (c == '-' || (c >= '0' && c <= '9')) return number();
    for (const auto& [word, kind, b] : {std::tuple<const char*, Json::Kind, bool>{"true", Json::Bool, true},
                                        {"false", Json::Bool, false}, {"null", Json::Null, false}}) {
      if (starts(word)) {
        at += std::char_traits<char>::length(word);
        Json j;
        j.kind = kind;
        j.b = b;
        skip();
        return j;
      }
    }
    fail(at, "No JSON value");
  }

  Json object() {
    Json j;
    j.kind = Json::Object;
    if (at < in.size() && in[at] == '}') {
      ++at;
      skip();
      return j;
    }
    for (;;) {
      const size_t key_at = at;
      if (at >= in.size() || in[at] != '"') fail(at, "No key");
      ++at;
      std::string key = string_body();
      skip();
      if (at >= in.size() || in[at] != ':') fail(at, "No :");
      ++at;
      skip();
      Json v = value();
      for (const auto& m : j.members)
        if (m.first == key) fail(key_at, "The key " + key + " twice");
      j.members.emplace_back(std::move(key), std::move(v));
      if (at < in.size() && in[at] == ',') {
        ++at;
        skip();
        continue;
      }
      if (at < in.size() && in[at] == '}') {
        ++at;
        skip();
        return j;
      }
      fail(at, "No , or } after a member");
    }
  }

  Json array() {
    Json j;
    j.kind = Json::Array;
    if (at < in.size() && in[at] == ']') {
      ++at;
      skip();
      return j;
    }
    for (;;) {
      j.items.push_back(value());
      if (at < in.size() && in[at] == ',') {
        ++at;
        skip();
        continue;
      }
      if (at < in.size() && in[at] == ']') {
        ++at;
        skip();
        return j;
      }
      fail(at, "No , or ] after an element");
    }
  }

  uint32_t hex4() {
    if (at + 4 > in.size()) fail(at, "A \\u escape without four hex digits");
    uint32_t code = 0;
    for (int k = 0; k < 4; ++k) {
      const char c = in[at + k];
      const int d = c >= '0' && c <= '9' ? c - '0' : c >= 'a' && c <= 'f' ? c - 'a' + 10 : c >= 'A' && c <= 'F' ? c - 'A' + 10 : -1;
      if (d < 0) fail(at, "A \\u escape without four hex digits");
      code = code * 16 + (uint32_t)d;
    }
    at += 4;
    return code;
  }

  // After the opening quote; leaves `at` after the closing one.
  std::string string_body() {
    std::string out;
    for (;;) {
      if (at >= in.size()) fail(at, "An unterminated string");
      const unsigned char c = (unsigned char)in[at];
      if (c == '"') {
        ++at;
        return out;
      }
      if (c < 0x20) fail(at, "A control character in a string");
      if (c != '\\') {
        out += (char)c;
        ++at;
        continue;
      }
      const size_t esc = ++at;
      if (at >= in.size()) fail(at, "An unknown escape");
      const char e = in[at++];
      switch (e) {
        case '"': out += '"'; break;
        case '\\': out += '\\'; break;
        case '/': out += '/'; break;
        case 'b': out += '\b'; break;
        case 'f': out += '\f'; break;
        case 'n': out += '\n'; break;
        case 'r': out += '\r'; break;
        case 't': out += '\t'; break;
        case 'u': {
          const size_t digits = at;
          const uint32_t code = hex4();
          if (code >= 0xD800 && code < 0xDC00) {
            if (!starts("\\u")) fail(at, "A lone surrogate");
            at += 2;
            const size_t low_at = at;
            const uint32_t low = hex4();
            if (low < 0xDC00 || low >= 0xE000) fail(low_at, "A lone surrogate");
            put_utf8(out, 0x10000 + ((code & 0x3FF) << 10) + (low & 0x3FF));
          } else if (code >= 0xDC00 && code < 0xE000) {
            fail(digits, "A lone surrogate");
          } else {
            put_utf8(out, code);
          }
          break;
        }
        default: fail(esc, "An unknown escape");
      }
    }
  }

  Json number() {
    std::string sign;
    if (in[at] == '-') {
      sign = "-";
      ++at;
    }
    const size_t start = at;
    while (at < in.size() && in[at] >= '0' && in[at] <= '9') ++at;
    const std::string digits = in.substr(start, at - start);
    if (digits.empty()) fail(start, "No digits");
    if (digits.size() > 1 && digits[0] == '0') fail(start, "A leading zero");
    if (at < in.size() && (in[at] == '.' || in[at] == 'e' || in[at] == 'E'))
      fail(at, "A number that is not an integer");
    Json j;
    j.kind = Json::Int;
    errno = 0;
    char* end = nullptr;
    const std::string text = sign + digits;
    j.i = std::strtoll(text.c_str(), &end, 10);
    if (errno == ERANGE) fail(start, "An integer past 64 bits");
    skip();
    return j;
  }
};

}  // namespace

std::string render_json(const Json& j) {
  std::string out;
  render(j, 0, out);
  return out + "\n";
}

Json parse_json(const std::string& text) {
  Reader r{text};
  r.skip();
  Json j = r.value();
  if (r.at != text.size()) r.fail(r.at, "Text after the value");
  return j;
}

}  // namespace fkh

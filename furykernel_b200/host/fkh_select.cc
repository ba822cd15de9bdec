// Variant spaces (src/FuryKernel/Variant.hs) and selections
// (src/FuryKernel/Selection.hs): the axes, points and names, the checks of
// a space, enumeration and its pruning, and the selection format with its
// validation, in the reference's words; and this target's GEMV family.
#include "fkh_select.h"

#include <algorithm>
#include <cinttypes>
#include <cstdio>

namespace fkh {

const char* kTargetName = "Cuda";

namespace {

bool lower_letters(const std::string& t) {
  if (t.empty()) return false;
  for (char c : t)
    if (c < 'a' || c > 'z') return false;
  return true;
}

bool all_digits(const std::string& t) {
  if (t.empty()) return false;
  for (char c : t)
    if (c < '0' || c > '9') return false;
  return true;
}

std::vector<std::string> split_on(const std::string& s, char sep) {
  std::vector<std::string> out;
  size_t at = 0;
  for (;;) {
    const size_t j = s.find(sep, at);
    out.push_back(s.substr(at, j == std::string::npos ? std::string::npos : j - at));
    if (j == std::string::npos) return out;
    at = j + 1;
  }
}

// Haskell's `show` of a Text: quoted, with escapes.
std::string show_text(const std::string& t) {
  std::string out = "\"";
  for (char c : t) {
    if (c == '"' || c == '\\') out += '\\';
    out += c;
  }
  return out + "\"";
}

uint64_t dim_of(const VShape& s, const std::string& d, bool& found) {
  for (const auto& [name, v] : s)
    if (name == d) {
      found = true;
      return v;
    }
  found = false;
  return 0;
}

std::string join(const std::vector<std::string>& xs, const std::string& sep) {
  std::string out;
  for (size_t i = 0; i < xs.size(); ++i) out += (i ? sep : "") + xs[i];
  return out;
}

}  // namespace

std::string hex64(uint64_t v) {
  char buf[24];
  std::snprintf(buf, sizeof buf, "0x%016" PRIx64, v);
  return buf;
}

std::vector<Point> points(const std::vector<Axis>& axes) {
  std::vector<Point> out{Point{}};
  for (const Axis& a : axes) {  // the first axis varies slowest
    std::vector<Point> next;
    for (const Point& p : out)
      for (uint64_t v : a.values) {
        Point q = p;
        q.emplace_back(a.prefix, v);
        next.push_back(std::move(q));
      }
    out = std::move(next);
  }
  return out;
}

std::string axis_key(const Point& p) {
  std::string out;
  for (size_t i = 0; i < p.size(); ++i) out += (i ? "_" : "") + p[i].first + std::to_string(p[i].second);
  return out;
}

std::string shape_key(const VShape& s) {
  std::string out;
  for (size_t i = 0; i < s.size(); ++i) out += (i ? "_" : "") + s[i].first + std::to_string(s[i].second);
  return out;
}

Point parse_axis_key(const std::vector<Axis>& axes, const std::string& key, const std::string& what) {
  const std::vector<std::string> parts = key.empty() ? std::vector<std::string>{} : split_on(key, '_');
  if (parts.size() != axes.size())
    throw Refusal(what + " " + key + " has " + std::to_string(parts.size()) + " parts for " +
                  std::to_string(axes.size()) + " axes.");
  Point p;
  for (size_t i = 0; i < axes.size(); ++i) {
    const Axis& a = axes[i];
    const std::string& part = parts[i];
    const bool prefixed = part.compare(0, a.prefix.size(), a.prefix) == 0;
    const std::string digits = prefixed ? part.substr(a.prefix.size()) : "";
    if (!prefixed || !all_digits(digits))
      throw Refusal(what + " " + key + " has " + part + " where " + a.name + " (" + a.prefix + ") belongs.");
    const uint64_t v = std::stoull(digits);
    if (std::to_string(v) != digits)
      throw Refusal(what + " " + key + " writes " + a.name + " " + std::to_string(v) + " as " + digits + ".");
    if (std::find(a.values.begin(), a.values.end(), v) == a.values.end())
      throw Refusal(what + " " + key + " gives " + a.name + " " + digits + ", which is not one of its values.");
    p.emplace_back(a.prefix, v);
  }
  return p;
}

std::string variant_name(const Space& sp, const VShape& s, const Point& p) {
  const std::string sk = shape_key(s), ak = axis_key(p);
  return sp.family + (sk.empty() ? "" : "_" + sk) + (ak.empty() ? "" : "_x_" + ak);
}

bool split_join(const std::function<bool(const std::string&)>& valid, const std::string& name, std::string& left,
                std::string& right) {
  for (size_t i = 0; i + 3 <= name.size(); ++i) {
    if (name.compare(i, 3, "_x_") != 0) continue;
    const std::string r = name.substr(i + 3);
    if (valid(r)) {
      left = name.substr(0, i);
      right = r;
      return true;
    }
  }
  return false;
}

bool variant_of_name(const Space& sp, const std::string& name, VShape& shape, Point& point) {
  point.clear();
  if (!sp.axes.empty()) {
    auto parses = [&](const std::string& k) {
      try {
        parse_axis_key(sp.axes, k);
        return true;
      } catch (const Refusal&) {
        return false;
      }
    };
    std::string left, key;
    if (!split_join(parses, name, left, key)) return false;
    point = parse_axis_key(sp.axes, key);
  }
  for (const VShape& s : sp.shapes)
    if (variant_name(sp, s, point) == name) {
      shape = s;
      return true;
    }
  return false;
}

std::vector<std::string> check_space(const Space& sp) {
  std::vector<std::string> out;
  if (sp.family.find("_x_") != std::string::npos)
    out.push_back("The family " + sp.family + " holds _x_, which joins a variant's name to its axis key.");
  for (const Axis& a : sp.axes)
    if (!lower_letters(a.prefix))
      out.push_back("The axis " + a.name + "'s prefix " + show_text(a.prefix) + " is not lowercase letters.");
  {
    std::map<std::string, std::vector<std::string>> by;  // prefixes in order, as a map lists them
    for (const Axis& a : sp.axes) by[a.prefix].push_back(a.name);
    for (const auto& [p, names] : by)
      if (names.size() > 1) out.push_back("The axes " + join(names, " and ") + " share the prefix " + p + ".");
  }
  for (const Axis& a : sp.axes)
    if (a.values.empty()) out.push_back("The axis " + a.name + " has no values.");
  for (const VShape& s : sp.shapes)
    for (const auto& [d, v] : s)
      if (!lower_letters(d))
        out.push_back("The class " + shape_key(s) + "'s dimension " + show_text(d) + " is not lowercase letters.");
  for (const VShape& s : sp.shapes) {
    std::map<std::string, size_t> count;
    for (const auto& [d, v] : s) ++count[d];
    for (const auto& [d, c] : count)
      if (c > 1) out.push_back("The class " + shape_key(s) + " gives " + d + " " + std::to_string(c) + " times.");
  }
  {
    std::map<std::string, size_t> count;
    for (const VShape& s : sp.shapes) ++count[shape_key(s)];
    for (const auto& [k, c] : count)
      if (c > 1) out.push_back("The class " + k + " is given " + std::to_string(c) + " times.");
  }
  for (const std::string& b : sp.batch)
    for (const VShape& s : sp.shapes) {
      bool found = false;
      dim_of(s, b, found);
      if (!found) out.push_back("The batch dimension " + b + " is not a dimension of the class " + shape_key(s) + ".");
    }
  return out;
}

std::vector<std::pair<Point, Outcome>> enumerate(const Space& sp, const VShape& s, uint64_t cores) {
  std::vector<std::pair<Point, Outcome>> out;
  std::map<uint64_t, Point> seen;  // kept kernels by identity
  for (const Point& p : points(sp.axes)) {
    Outcome o = sp.consider(s, p, cores);
    if (o.kind == Outcome::Kept) {
      auto it = seen.find(o.hash);
      if (it != seen.end()) {
        Outcome dup;
        dup.kind = Outcome::SameAs;
        dup.same_as = it->second;
        out.emplace_back(p, dup);
        continue;
      }
      seen.emplace(o.hash, p);
    }
    out.emplace_back(p, o);
  }
  return out;
}

// ---------------------------------------------------------------------------
// Selections

std::string render_selection(const Selection& s) {
  std::vector<std::pair<std::string, Json>> classes;
  for (const auto& [c, p] : s.classes)
    classes.emplace_back(c, Json::obj({{"variant", Json::str(p.axes)}, {"ir_hash", Json::str(hex64(p.hash))}}));
  return render_json(Json::obj({{"format", Json::str("furykernel-selection")},
                                {"version", Json::num(1)},
                                {"family", Json::str(s.family)},
                                {"target", Json::str(s.target)},
                                {"profile", Json::obj({{"cores", Json::num((int64_t)s.cores)}})},
                                {"classes", Json::obj(std::move(classes))}}));
}

Selection parse_selection(const std::string& text) {
  Json j = parse_json(text);
  if (j.kind != Json::Object) throw Refusal("A selection is a JSON object.");
  auto field = [&](const std::string& name) -> const Json& {
    for (const auto& m : j.members)
      if (m.first == name) return m.second;
    throw Refusal("The field " + name + " is missing.");
  };
  auto wrong = [](const std::string& name) { return Refusal("The field " + name + " has the wrong type."); };
  const Json& format = field("format");
  if (format.kind != Json::String) throw wrong("format");
  if (format.s != "furykernel-selection")
    throw Refusal("The format is " + format.s + ", not furykernel-selection.");
  const Json& version = field("version");
  if (version.kind != Json::Int) throw wrong("version");
  if (version.i != 1)
    throw Refusal("Version " + std::to_string(version.i) + " of the format; this reads version 1.");
  std::vector<std::string> unknown;
  for (const auto& m : j.members)
    if (m.first != "format" && m.first != "version" && m.first != "family" && m.first != "target" &&
        m.first != "profile" && m.first != "classes")
      unknown.push_back("An unknown field: " + m.first + ".");
  if (!unknown.empty()) throw Refusal(join(unknown, "\n"));
  Selection s;
  const Json& family = field("family");
  if (family.kind != Json::String) throw wrong("family");
  s.family = family.s;
  const Json& target = field("target");
  if (target.kind != Json::String) throw wrong("target");
  s.target = target.s;
  const Json& profile = field("profile");
  if (profile.kind != Json::Object || profile.members.size() != 1 || profile.members[0].first != "cores" ||
      profile.members[0].second.kind != Json::Int || profile.members[0].second.i < 0)
    throw wrong("profile");
  s.cores = (uint64_t)profile.members[0].second.i;
  const Json& classes = field("classes");
  if (classes.kind != Json::Object) throw wrong("classes");
  for (const auto& [c, v] : classes.members) {
    if (v.kind != Json::Object || v.members.size() != 2 || v.members[0].first != "variant" ||
        v.members[0].second.kind != Json::String || v.members[1].first != "ir_hash" ||
        v.members[1].second.kind != Json::String)
      throw wrong("classes");
    const std::string& h = v.members[1].second.s;  // 0x and 16 lowercase hex digits, as hex64 writes them
    if (h.size() != 18 || h.compare(0, 2, "0x") != 0) throw wrong("classes");
    uint64_t hash = 0;
    for (size_t i = 2; i < 18; ++i) {
      const char d = h[i];
      const int x = d >= '0' && d <= '9' ? d - '0' : d >= 'a' && d <= 'f' ? d - 'a' + 10 : -1;
      if (x < 0) throw wrong("classes");
      hash = hash * 16 + (uint64_t)x;
    }
    s.classes[c] = Pick{v.members[0].second.s, hash};
  }
  return s;
}

std::vector<Point> validate_selection(uint64_t cores, const std::string& target, const Space& sp,
                                      const Selection& sel) {
  std::vector<std::string> problems = check_space(sp);
  if (sel.cores != cores)
    problems.push_back("The selection was made for a GPU of " + std::to_string(sel.cores) + " cores, not " +
                       std::to_string(cores) + ".");
  if (sel.family != sp.family)
    problems.push_back("The selection is for the family " + sel.family + ", not " + sp.family + ".");
  if (sel.target != target)
    problems.push_back("The selection is for the target " + sel.target + ", not " + target + ".");
  std::vector<std::string> keys;
  for (const VShape& s : sp.shapes) keys.push_back(shape_key(s));
  for (const std::string& k : keys)
    if (!sel.classes.count(k)) problems.push_back("No variant for the class " + k + ".");
  for (const auto& [c, p] : sel.classes)
    if (std::find(keys.begin(), keys.end(), c) == keys.end())
      problems.push_back("The class " + c + " is not one of the family's.");
  // Each class's pick, in the space's order.
  struct Picked {
    const VShape* shape;
    bool ok;
    Point point;
  };
  std::vector<Picked> picked;
  for (const VShape& s : sp.shapes) {
    auto it = sel.classes.find(shape_key(s));
    if (it == sel.classes.end()) continue;
    Picked pk{&s, false, {}};
    try {
      pk.point = parse_axis_key(sp.axes, it->second.axes, "The class " + shape_key(s) + "'s axis key");
      const std::string name = variant_name(sp, s, pk.point);
      const Outcome o = sp.consider(s, pk.point, cores);
      switch (o.kind) {
        case Outcome::Kept:
          if (o.hash != it->second.hash)
            problems.push_back(name + " was picked as the kernel of IR hash " + hex64(it->second.hash) +
                               ", and is now " + hex64(o.hash) + ".");
          else
            pk.ok = true;
          break;
        case Outcome::Illegal: problems.push_back(name + " is illegal: " + join(o.reasons, " ")); break;
        case Outcome::Indivisible:
          problems.push_back(name + " does not divide its class: " + join(o.reasons, " "));
          break;
        case Outcome::TooFewGroups:
          problems.push_back(name + " launches " + std::to_string(o.groups) + " threadgroups, fewer than twice the " +
                             std::to_string(cores) + " cores.");
          break;
        case Outcome::SameAs:
          problems.push_back(name + " is the same kernel as " + axis_key(o.same_as) + ".");
          break;
      }
    } catch (const Refusal& e) {
      problems.push_back(e.what());
    }
    picked.push_back(pk);
  }
  // Classes that differ only in batch dimensions agree on the axes that
  // order a reduction.
  auto unbatched = [&](const VShape& s) {
    VShape out;
    for (const auto& d : s)
      if (std::find(sp.batch.begin(), sp.batch.end(), d.first) == sp.batch.end()) out.push_back(d);
    return out;
  };
  auto order_of = [&](const Point& p) {
    Point out;
    for (const auto& v : p)
      for (const Axis& a : sp.axes)
        if (a.order && a.prefix == v.first) out.push_back(v);
    return out;
  };
  for (size_t i = 0; i < picked.size(); ++i)
    for (size_t j = i + 1; j < picked.size(); ++j) {
      if (!picked[i].ok || !picked[j].ok) continue;
      if (unbatched(*picked[i].shape) != unbatched(*picked[j].shape)) continue;
      const Point pa = order_of(picked[i].point), pb = order_of(picked[j].point);
      if (pa != pb)
        problems.push_back("The classes " + shape_key(*picked[i].shape) + " and " + shape_key(*picked[j].shape) +
                           " differ only in batch size, and order reductions differently: " + axis_key(pa) +
                           " against " + axis_key(pb) + ".");
    }
  if (!problems.empty()) throw Refusal(join(problems, "\n"));
  std::vector<Point> out;
  for (const Picked& pk : picked) out.push_back(pk.point);
  return out;
}

// ---------------------------------------------------------------------------
// This target's GEMV family

namespace {

// Bumped when a GEMV kernel's arithmetic or launch changes, so that
// committed picks name the kernels they were measured on.
constexpr const char* kGemvRevision = "gemv kernels 1";

uint64_t fnv(const std::string& s) {
  uint64_t h = 0xcbf29ce484222325ULL;
  for (unsigned char c : s) {
    h ^= c;
    h *= 0x100000001b3ULL;
  }
  return h;
}

}  // namespace

Space gemv_space(const std::vector<VShape>& classes) {
  Space sp;
  sp.family = "gemv";
  sp.axes = {Axis{"split_k", "s", {1, 2, 4, 8}, true}};
  sp.shapes = classes;
  sp.batch = {"m"};
  sp.consider = [](const VShape& s, const Point& p, uint64_t cores) {
    Outcome o;
    bool fn = false, fk = false, fm = false;
    const uint64_t n = dim_of(s, "n", fn), k = dim_of(s, "k", fk), m = dim_of(s, "m", fm);
    uint64_t split = 1;
    for (const auto& v : p)
      if (v.first == "s") split = v.second;
    if (!fn || !fk || !fm || n == 0 || k == 0 || m == 0) {
      o.kind = Outcome::Illegal;
      o.reasons = {"A GEMV class gives n, k and m, each at least 1."};
      return o;
    }
    if (m > 64 || n > 1048576 || k > 65536) {
      o.kind = Outcome::Illegal;
      o.reasons = {"The table's GEMVs take n up to 1048576, k up to 65536 and batches of up to 64 rows."};
      return o;
    }
    if (k % 4 != 0) {
      o.kind = Outcome::Indivisible;
      o.reasons = {"k " + std::to_string(k) + " is not a multiple of the pack of 4."};
      return o;
    }
    // The kernel the runtime runs for (m, s), and its independent work:
    // rows (a warp each) for the streaming kernel, 4-row groups for the
    // batched one, 8-warp blocks for the chunked one.
    std::string kernel;
    uint64_t units = 0;
    if (m <= 4 && m * k * 4 <= 200 * 1024) {
      kernel = "stream";
      units = n;
    } else if (split == 1) {
      kernel = "batch";
      units = (n + 3) / 4;
    } else {
      kernel = "chunk";
      units = (n + 8 / split - 1) / (8 / split);
    }
    if (units < 2 * cores) {
      o.kind = Outcome::TooFewGroups;
      o.groups = units;
      return o;
    }
    o.kind = Outcome::Kept;
    o.groups = units;
    o.hash = fnv(std::string(kGemvRevision) + "\nkernel " + kernel + "\nn " + std::to_string(n) + "\nk " +
                 std::to_string(k) + "\nm " + std::to_string(m) + "\nsplit " + std::to_string(split) + "\n");
    return o;
  };
  return sp;
}

}  // namespace fkh

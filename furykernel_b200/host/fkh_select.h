// Variant spaces and selections of the host library: JSON
// (src/FuryKernel/Json.hs), a family's axes, points, shape classes and
// their names (src/FuryKernel/Variant.hs), and the committed selections
// that pick one variant a class (src/FuryKernel/Selection.hs); and this
// target's GEMV family, whose one axis is the split-K.
#pragma once

#include <cstdint>
#include <functional>
#include <map>
#include <string>
#include <utility>
#include <vector>

#include "fkh.h"

namespace fkh {

struct Json {
  enum Kind { Null, Bool, Int, String, Array, Object } kind = Null;
  bool b = false;
  int64_t i = 0;
  std::string s;
  std::vector<Json> items;
  std::vector<std::pair<std::string, Json>> members;
  static Json str(std::string v) {
    Json j;
    j.kind = String;
    j.s = std::move(v);
    return j;
  }
  static Json num(int64_t v) {
    Json j;
    j.kind = Int;
    j.i = v;
    return j;
  }
  static Json obj(std::vector<std::pair<std::string, Json>> m) {
    Json j;
    j.kind = Object;
    j.members = std::move(m);
    return j;
  }
  bool operator==(const Json& o) const {
    return kind == o.kind && b == o.b && i == o.i && s == o.s && items == o.items && members == o.members;
  }
};
std::string render_json(const Json& j);
Json parse_json(const std::string& text);  // throws Refusal with the place

// ---------------------------------------------------------------------------
// Axes, points, classes (Variant.hs)

struct Axis {
  std::string name, prefix;
  std::vector<uint64_t> values;
  bool order = false;  // decides the order of a reduction
};
using Point = std::vector<std::pair<std::string, uint64_t>>;  // by prefix, in the axes' order
using VShape = std::vector<std::pair<std::string, uint64_t>>;  // a class's dimensions by name

std::vector<Point> points(const std::vector<Axis>& axes);
std::string axis_key(const Point& p);
std::string shape_key(const VShape& s);
// The point an axis key names, or why not (as `what` names the key).
Point parse_axis_key(const std::vector<Axis>& axes, const std::string& key,
                     const std::string& what = "The axis key");

// What pruning made of a point.
struct Outcome {
  enum Kind { Kept, Illegal, Indivisible, TooFewGroups, SameAs } kind = Kept;
  uint64_t groups = 0;               // Kept, TooFewGroups: threadgroups of the launch
  std::vector<std::string> reasons;  // Illegal, Indivisible
  Point same_as;                     // SameAs
  uint64_t hash = 0;                 // Kept: the variant's kernel identity
};

struct Space {
  std::string family;
  std::vector<Axis> axes;
  std::vector<VShape> shapes;
  std::vector<std::string> batch;  // the dimensions that are batch sizes
  // A point for a class, pruned by everything but duplicates, on a GPU of
  // `cores` multiprocessors.
  std::function<Outcome(const VShape&, const Point&, uint64_t cores)> consider;
};

std::string variant_name(const Space& sp, const VShape& s, const Point& p);
// A name joined with _x_, split at the first _x_ whose right side is valid.
bool split_join(const std::function<bool(const std::string&)>& valid, const std::string& name, std::string& left,
                std::string& right);
bool variant_of_name(const Space& sp, const std::string& name, VShape& shape, Point& point);
std::vector<std::string> check_space(const Space& sp);
// Every point of a class and its outcome, duplicates (same kernel
// identity as a kept point) marked.
std::vector<std::pair<Point, Outcome>> enumerate(const Space& sp, const VShape& s, uint64_t cores);

// ---------------------------------------------------------------------------
// Selections (Selection.hs)

struct Pick {
  std::string axes;  // the variant's axis key
  uint64_t hash = 0;
  bool operator==(const Pick& o) const { return axes == o.axes && hash == o.hash; }
};
struct Selection {
  std::string family, target;
  uint64_t cores = 0;
  std::map<std::string, Pick> classes;  // by shape key, written in key order
};
std::string render_selection(const Selection& s);
Selection parse_selection(const std::string& text);  // throws Refusal: the problems, one a line
// The selected point of every class, in the space's class order; throws
// Refusal with every problem, one a line.
std::vector<Point> validate_selection(uint64_t cores, const std::string& target, const Space& sp, const Selection& sel);
std::string hex64(uint64_t v);

// ---------------------------------------------------------------------------
// This target's GEMV family: classes n_k_m (m the batch), one axis, the
// split-K s (an order axis). The kernel a point runs follows from m and s,
// as the runtime picks it: the streaming kernel for batches of up to 4 rows
// whose x fits its shared memory, the batched one for up to 64 rows at
// split 1, the chunked one otherwise (splits 1, 2, 4, 8).
Space gemv_space(const std::vector<VShape>& classes);
extern const char* kTargetName;  // "Cuda"

}  // namespace fkh

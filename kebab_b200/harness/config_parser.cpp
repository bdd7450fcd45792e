// YAML-subset reader and the ConfigParser getters (see config_parser.h).
#include "config_parser.h"

#include <algorithm>
#include <cctype>
#include <fstream>
#include <sstream>
#include <stdexcept>

namespace kebab {
namespace config {

const Node* Node::child(const std::string& key) const {
  if (kind != MAP) return nullptr;
  for (const auto& kv : map)
    if (kv.first == key) return kv.second.get();
  return nullptr;
}

namespace {

struct Line {
  int indent;
  std::string text;  // without indentation and comments, right-trimmed
  int number;
};

std::string rtrim(const std::string& s) {
  size_t e = s.find_last_not_of(" \t\r");
  return e == std::string::npos ? "" : s.substr(0, e + 1);
}
std::string trim(const std::string& s) {
  size_t b = s.find_first_not_of(" \t\r");
  return b == std::string::npos ? "" : rtrim(s.substr(b));
}

// Removes a trailing comment that is not inside quotes.
std::string strip_comment(const std::string& s) {
  char q = 0;
  for (size_t i = 0; i < s.size(); ++i) {
    char c = s[i];
    if (q) {
      if (c == q) q = 0;
    } else if (c == '"' || c == '\'') {
      q = c;
    } else if (c == '#' && (i == 0 || s[i - 1] == ' ' || s[i - 1] == '\t')) {
      return s.substr(0, i);
    }
  }
  return s;
}

std::string unquote(const std::string& s) {
  if (s.size() >= 2 && ((s.front() == '"' && s.back() == '"') || (s.front() == '\'' && s.back() == '\'')))
    return s.substr(1, s.size() - 2);
  return s;
}

std::shared_ptr<Node> scalar(const std::string& s) {
  auto n = std::make_shared<Node>();
  n->kind = Node::SCALAR;
  n->scalar = unquote(trim(s));
  return n;
}

// Flow sequence "[a, [b, c], d]".
std::shared_ptr<Node> parse_flow(const std::string& s, size_t& i, int line) {
  auto n = std::make_shared<Node>();
  n->kind = Node::SEQ;
  if (s[i] != '[') throw std::runtime_error("line " + std::to_string(line) + ": expected '['");
  ++i;
  std::string cur;
  auto flush = [&] {
    std::string t = trim(cur);
    if (!t.empty()) n->seq.push_back(scalar(t));
    cur.clear();
  };
  while (i < s.size()) {
    char c = s[i];
    if (c == '[') {
      n->seq.push_back(parse_flow(s, i, line));
      continue;
    }
    if (c == ']') {
      flush();
      ++i;
      return n;
    }
    if (c == ',') {
      flush();
      ++i;
      continue;
    }
    cur += c;
    ++i;
  }
  throw std::runtime_error("line " + std::to_string(line) + ": unterminated '['");
}

std::shared_ptr<Node> value_node(const std::string& v, int line) {
  std::string t = trim(v);
  if (!t.empty() && t[0] == '[') {
    size_t i = 0;
    return parse_flow(t, i, line);
  }
  return scalar(t);
}

class Parser {
 public:
  explicit Parser(std::vector<Line> lines) : lines_(std::move(lines)) {}
  std::shared_ptr<Node> parse() {
    if (lines_.empty()) return std::make_shared<Node>();
    return block(lines_[0].indent);
  }

 private:
  std::vector<Line> lines_;
  size_t pos_ = 0;

  std::shared_ptr<Node> block(int indent) {
    const Line& first = lines_[pos_];
    if (first.text.rfind("- ", 0) == 0 || first.text == "-") return sequence(indent);
    return mapping(indent);
  }

  std::shared_ptr<Node> sequence(int indent) {
    auto n = std::make_shared<Node>();
    n->kind = Node::SEQ;
    while (pos_ < lines_.size() && lines_[pos_].indent == indent &&
           (lines_[pos_].text.rfind("- ", 0) == 0 || lines_[pos_].text == "-")) {
      const Line l = lines_[pos_++];
      std::string item = l.text == "-" ? "" : trim(l.text.substr(2));
      if (item.empty()) {
        if (pos_ < lines_.size() && lines_[pos_].indent > indent) n->seq.push_back(block(lines_[pos_].indent));
        else n->seq.push_back(std::make_shared<Node>());
      } else if (item[0] != '[' && item.find(": ") != std::string::npos) {
        // "- key: value" starts an inline mapping item.
        auto m = std::make_shared<Node>();
        m->kind = Node::MAP;
        size_t c = item.find(": ");
        m->map.emplace_back(trim(item.substr(0, c)), value_node(item.substr(c + 2), l.number));
        while (pos_ < lines_.size() && lines_[pos_].indent > indent) {
          auto rest = mapping(lines_[pos_].indent);
          for (auto& kv : rest->map) m->map.push_back(kv);
        }
        n->seq.push_back(m);
      } else {
        n->seq.push_back(value_node(item, l.number));
      }
    }
    return n;
  }

  std::shared_ptr<Node> mapping(int indent) {
    auto n = std::make_shared<Node>();
    n->kind = Node::MAP;
    while (pos_ < lines_.size() && lines_[pos_].indent == indent) {
      const Line l = lines_[pos_];
      if (l.text.rfind("- ", 0) == 0) break;
      size_t c = l.text.find(':');
      if (c == std::string::npos)
        throw std::runtime_error("line " + std::to_string(l.number) + ": expected 'key: value'");
      std::string key = unquote(trim(l.text.substr(0, c)));
      std::string rest = trim(l.text.substr(c + 1));
      ++pos_;
      if (!rest.empty()) {
        n->map.emplace_back(key, value_node(rest, l.number));
      } else if (pos_ < lines_.size() && (lines_[pos_].indent > indent ||
                                          (lines_[pos_].indent == indent && lines_[pos_].text.rfind("- ", 0) == 0))) {
        n->map.emplace_back(key, block(lines_[pos_].indent));
      } else {
        n->map.emplace_back(key, std::make_shared<Node>());
      }
    }
    if (pos_ < lines_.size() && lines_[pos_].indent > indent)
      throw std::runtime_error("line " + std::to_string(lines_[pos_].number) + ": unexpected indentation");
    return n;
  }
};

const Node* walk(const Node* root, const std::string& dotted) {
  const Node* n = root;
  size_t start = 0;
  while (n) {
    size_t dot = dotted.find('.', start);
    std::string k = dotted.substr(start, dot == std::string::npos ? std::string::npos : dot - start);
    n = n->child(k);
    if (dot == std::string::npos) break;
    start = dot + 1;
  }
  return n;
}

bool to_int(const std::string& s, long long* out) {
  if (s.empty()) return false;
  char* end = nullptr;
  long long v = std::strtoll(s.c_str(), &end, 0);
  if (*end) return false;
  *out = v;
  return true;
}

}  // namespace

std::shared_ptr<Node> parse_yaml(const std::string& text) {
  std::vector<Line> lines;
  std::istringstream in(text);
  std::string raw;
  int number = 0;
  while (std::getline(in, raw)) {
    ++number;
    if (raw.find('\t') != std::string::npos && raw.find_first_not_of(" \t") != std::string::npos &&
        raw.find('\t') < raw.find_first_not_of(" \t"))
      throw std::runtime_error("line " + std::to_string(number) + ": tabs are not allowed for indentation");
    std::string s = rtrim(strip_comment(raw));
    if (trim(s).empty() || trim(s) == "---") continue;
    int indent = (int)s.find_first_not_of(' ');
    lines.push_back({indent, s.substr(indent), number});
  }
  Parser p(std::move(lines));
  return p.parse();
}

ConfigParser::ConfigParser(const std::string& path) { reload(path); }

ConfigParser& ConfigParser::getInstance(const std::string& config_path) {
  static ConfigParser instance(config_path);
  return instance;
}

void ConfigParser::reload(const std::string& config_path) {
  if (!config_path.empty()) path_ = config_path;
  std::ifstream f(path_);
  if (!f) throw std::runtime_error("cannot open config file: " + path_);
  std::stringstream ss;
  ss << f.rdbuf();
  root_ = parse_yaml(ss.str());
}

const Node* ConfigParser::find(const std::string& dotted) const { return walk(root_.get(), dotted); }

std::string ConfigParser::getString(const std::string& k, const std::string& def) const {
  const Node* n = find(k);
  return (n && n->kind == Node::SCALAR) ? n->scalar : def;
}

long long ConfigParser::getInt(const std::string& k, long long def) const {
  const Node* n = find(k);
  long long v;
  return (n && n->kind == Node::SCALAR && to_int(n->scalar, &v)) ? v : def;
}

bool ConfigParser::getBool(const std::string& k, bool def) const {
  const Node* n = find(k);
  if (!n || n->kind != Node::SCALAR) return def;
  std::string s = n->scalar;
  std::transform(s.begin(), s.end(), s.begin(), [](unsigned char c) { return (char)std::tolower(c); });
  if (s == "true" || s == "yes" || s == "on" || s == "1") return true;
  if (s == "false" || s == "no" || s == "off" || s == "0") return false;
  return def;
}

std::vector<std::string> ConfigParser::getStrings(const std::string& k, const std::vector<std::string>& def) const {
  const Node* n = find(k);
  if (!n || n->kind != Node::SEQ) return def;
  std::vector<std::string> out;
  for (const auto& e : n->seq) {
    if (e->kind != Node::SCALAR) return def;
    out.push_back(e->scalar);
  }
  return out;
}

std::vector<long long> ConfigParser::getInts(const std::string& k, const std::vector<long long>& def) const {
  const Node* n = find(k);
  if (!n || n->kind != Node::SEQ) return def;
  std::vector<long long> out;
  for (const auto& e : n->seq) {
    long long v;
    if (e->kind != Node::SCALAR || !to_int(e->scalar, &v)) return def;
    out.push_back(v);
  }
  return out;
}

static std::vector<int> to_int_vec(const std::vector<long long>& v) { return std::vector<int>(v.begin(), v.end()); }

std::string ConfigParser::getBuildMode() const { return getString("build.mode", "release"); }
std::string ConfigParser::getOptimizationLevel() const { return getString("build.optimization", "O3"); }
std::string ConfigParser::getCudaArch() const { return getString("build.cuda_arch", "auto"); }
int ConfigParser::getWarmupRuns() const { return (int)getInt("benchmark.warmup_runs", 10); }
int ConfigParser::getMeasurementRuns() const { return (int)getInt("benchmark.measurement_runs", 100); }
std::vector<int> ConfigParser::getBatchSizes() const {
  return to_int_vec(getInts("benchmark.batch_sizes", {256, 512, 1024, 2048, 4096}));
}
std::vector<std::string> ConfigParser::getDataTypes() const { return getStrings("benchmark.data_types", {"float32"}); }
std::vector<std::string> ConfigParser::getProfilingMetrics() const { return getStrings("profiling.ncu_metrics", {}); }
std::vector<std::string> ConfigParser::getProfilingSections() const { return getStrings("profiling.sections", {}); }

bool ConfigParser::isOperatorEnabled(const std::string& op) const {
  return getBool("operators." + op + ".enabled", true);
}
std::vector<int> ConfigParser::getOperatorSizes(const std::string& op) const {
  return to_int_vec(getInts("operators." + op + ".sizes", {}));
}
std::vector<int> ConfigParser::getOperatorMatrixSizes(const std::string& op) const {
  return to_int_vec(getInts("operators." + op + ".matrix_sizes", {}));
}
std::vector<std::string> ConfigParser::getOperatorModes(const std::string& op) const {
  return getStrings("operators." + op + ".modes", {"NT"});
}
std::vector<std::string> ConfigParser::getOperatorPrecisions(const std::string& op) const {
  return getStrings("operators." + op + ".precisions", {"float16"});
}
std::vector<std::string> ConfigParser::getOperatorImpls(const std::string& op) const {
  auto v = getStrings("operators." + op + ".impl", {});
  if (!v.empty()) return v;
  std::string one = getString("operators." + op + ".impl", "");
  if (!one.empty()) return {one};
  return {"cute"};
}
std::string ConfigParser::getOperatorImpl(const std::string& op) const { return getOperatorImpls(op)[0]; }
std::vector<int> ConfigParser::getOperatorVersions(const std::string& op) const {
  auto v = getInts("operators." + op + ".versions", {});
  if (!v.empty()) return to_int_vec(v);
  long long one = getInt("operators." + op + ".version", -1);
  if (one >= 0) return {(int)one};
  return {1};
}
int ConfigParser::getOperatorVersion(const std::string& op) const { return getOperatorVersions(op)[0]; }
std::string ConfigParser::getOperatorInitMethod(const std::string& op) const {
  return getString("operators." + op + ".init_method", "rand-rand");
}
bool ConfigParser::getOperatorVerbose(const std::string& op) const {
  return getBool("operators." + op + ".verbose", false);
}
int ConfigParser::getOperatorGpuId(const std::string& op) const {
  return (int)getInt("operators." + op + ".gpu_id", 0);
}
std::vector<std::vector<long long>> ConfigParser::getOperatorShapes(const std::string& op) const {
  std::vector<std::vector<long long>> out;
  const Node* n = find("operators." + op + ".shapes");
  if (!n || n->kind != Node::SEQ) return out;
  for (const auto& e : n->seq) {
    if (e->kind != Node::SEQ || e->seq.size() != 3) continue;
    std::vector<long long> s;
    for (const auto& x : e->seq) {
      long long v;
      if (x->kind == Node::SCALAR && to_int(x->scalar, &v)) s.push_back(v);
    }
    if (s.size() == 3) out.push_back(s);
  }
  return out;
}
unsigned ConfigParser::getOperatorSeed(const std::string& op) const {
  return (unsigned)getInt("operators." + op + ".seed", 42);
}

}  // namespace config
}  // namespace kebab

// Configuration reader for the benchmark harness: the same getters, keys and
// defaults as the reference's ConfigParser (kebab/include/kebab/config/
// config_parser.h:17-91, kebab/lib/common/config_parser.cpp:115-396), backed
// by a small YAML-subset reader instead of yaml-cpp (which this build does
// not depend on). Supported YAML: block mappings, block sequences ("- x"),
// flow sequences ("[a, b]", nested one level), plain / quoted scalars,
// comments. Keys are addressed with dots ("operators.gemm.versions").
#pragma once

#include <map>
#include <memory>
#include <string>
#include <vector>

namespace kebab {
namespace config {

struct Node {
  enum Kind { NIL, SCALAR, SEQ, MAP } kind = NIL;
  std::string scalar;
  std::vector<std::shared_ptr<Node>> seq;
  std::vector<std::pair<std::string, std::shared_ptr<Node>>> map;  // insertion order
  const Node* child(const std::string& key) const;
};

// Parses YAML text; throws std::runtime_error with a line number on errors.
std::shared_ptr<Node> parse_yaml(const std::string& text);

class ConfigParser {
 public:
  // Loads `path` (reads it once; reload() re-reads).
  explicit ConfigParser(const std::string& path = "config.yaml");
  static ConfigParser& getInstance(const std::string& config_path = "config.yaml");

  std::string getBuildMode() const;          // build.mode, "release"
  std::string getOptimizationLevel() const;  // build.optimization, "O3"
  std::string getCudaArch() const;           // build.cuda_arch, "auto"
  int getWarmupRuns() const;                 // benchmark.warmup_runs, 10
  int getMeasurementRuns() const;            // benchmark.measurement_runs, 100
  std::vector<int> getBatchSizes() const;
  std::vector<std::string> getDataTypes() const;
  std::vector<std::string> getProfilingMetrics() const;
  std::vector<std::string> getProfilingSections() const;

  bool isOperatorEnabled(const std::string& op) const;                          // enabled, true
  std::vector<int> getOperatorSizes(const std::string& op) const;               // sizes
  std::vector<int> getOperatorMatrixSizes(const std::string& op) const;         // matrix_sizes
  std::vector<std::string> getOperatorModes(const std::string& op) const;       // modes, {"NT"}
  std::vector<std::string> getOperatorPrecisions(const std::string& op) const;  // precisions, {"float16"}
  std::string getOperatorImpl(const std::string& op) const;                     // first impl, "cute"
  std::vector<std::string> getOperatorImpls(const std::string& op) const;       // impl (list or scalar)
  int getOperatorVersion(const std::string& op) const;                          // first version, 1
  std::vector<int> getOperatorVersions(const std::string& op) const;            // versions / version
  std::string getOperatorInitMethod(const std::string& op) const;               // init_method, "rand-rand"
  bool getOperatorVerbose(const std::string& op) const;                         // verbose, false
  int getOperatorGpuId(const std::string& op) const;                            // gpu_id, 0

  // Keys added by this build (absent in the reference's schema):
  //   operators.<op>.shapes: [[M, N, K], ...]  non-square problems
  //   operators.<op>.seed:   RNG seed (default 42, the reference's fixed seed)
  std::vector<std::vector<long long>> getOperatorShapes(const std::string& op) const;
  unsigned getOperatorSeed(const std::string& op) const;

  void reload(const std::string& config_path = "");
  std::string getConfigPath() const { return path_; }

  // Generic access.
  const Node* find(const std::string& dotted) const;
  std::string getString(const std::string& dotted, const std::string& def) const;
  long long getInt(const std::string& dotted, long long def) const;
  bool getBool(const std::string& dotted, bool def) const;
  std::vector<std::string> getStrings(const std::string& dotted, const std::vector<std::string>& def) const;
  std::vector<long long> getInts(const std::string& dotted, const std::vector<long long>& def) const;

 private:
  std::string path_;
  std::shared_ptr<Node> root_;
};

}  // namespace config
}  // namespace kebab

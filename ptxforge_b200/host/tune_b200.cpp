// tune_b200.cpp -- PTXForge's tuner CLI driving the sm_100a backend.
//
// Built inside the PTXForge include tree (ptxforge/search.hpp, advisors, trace writer) and linked
// against libpf_b200.so; the search loop, search space, trace schema and correctness gate are the
// reference's own, only the Runner differs.  Subcommands:
//
//   tune     like `ptxforge-tune tune` (core/src/main.cpp:95-117) with a B200Runner:
//            tune --dtype bf16 --M 8192 --N 8192 --K 8192 --gpus 1 --budget 30 --advisor rules --out t.json
//            --fanout G measures up to G candidates per round, each on its own GPU(s) (tune_fanout.hpp);
//            G = 1 (the default) is the reference's tune() unchanged
//   measure  gate and time one config (like `ptxforge-tune bench`, core/src/main.cpp:224-238), one
//            JSON line, exit 4 if the trial failed:
//            measure --dtype bf16 --BM 128 --BN 256 --BK 32 --TM 4 --TN 16 --PAD 0 --M ... --gpus 2
//   gpus     the B200 row this runner reports (hw.hpp has none)
#include <cstdio>
#include <cstdlib>
#include <filesystem>
#include <fstream>
#include <map>
#include <string>

#include "ptxforge/search.hpp"
#include "ptxforge_b200/b200_runner.hpp"
#include "ptxforge_b200/tune_fanout.hpp"

using namespace ptxforge;

namespace {

struct Args {
  std::map<std::string, std::string> kv;
  static Args parse(int argc, char **argv, int from) {
    Args a;
    for (int i = from; i < argc; ++i) {
      std::string k = argv[i];
      if (k.rfind("--", 0) != 0) throw std::runtime_error("unexpected argument '" + k + "'");
      if (i + 1 >= argc) throw std::runtime_error("missing value for " + k);
      a.kv[k.substr(2)] = argv[++i];
    }
    return a;
  }
  std::string get(const std::string &k, const std::string &d) const {
    auto it = kv.find(k);
    return it == kv.end() ? d : it->second;
  }
  int geti(const std::string &k, int d) const {
    auto it = kv.find(k);
    return it == kv.end() ? d : std::stoi(it->second);
  }
};

pf_dtype parse_dtype(const std::string &s) {
  if (s == "f32") return PF_F32;
  if (s == "f32_3xtf32") return PF_F32_3XTF32;
  if (s == "bf16") return PF_BF16;
  if (s == "e4m3") return PF_E4M3;
  throw std::runtime_error("unknown dtype '" + s + "' (f32|f32_3xtf32|bf16|e4m3)");
}

B200Runner::Options runner_options(const Args &a) {
  B200Runner::Options o;
  o.dtype = parse_dtype(a.get("dtype", "bf16"));
  o.device = a.geti("device", 0);
  o.gpus = a.geti("gpus", 1);
  o.warmup = a.geti("warmup", 5);
  o.iters = a.geti("iters", 20);
  o.reps = a.geti("reps", 5);
  o.samples = a.geti("samples", 512);
  o.seed = static_cast<uint64_t>(a.geti("seed", 0));
  o.root = a.get("root", ".");
  o.nvcc = a.get("nvcc", "nvcc");
  o.workdir = a.get("workdir", "build/kernels");
  o.jit = a.get("jit", "1") != "0";
  o.cublas = a.get("cublas", "1") != "0";
  o.fanout = a.geti("fanout", 1);
  return o;
}

Problem problem_of(const Args &a) { return Problem{a.geti("M", 2048), a.geti("N", 2048), a.geti("K", 2048)}; }

json::Value measurement_json(const Measurement &m) {
  json::Value j = json::Value::object();
  j.set("ok", m.ok).set("error", m.ok ? json::Value() : json::Value(m.error));
  j.set("gflops", m.gflops ? json::Value(*m.gflops) : json::Value()).set("ms", m.ms ? json::Value(*m.ms) : json::Value());
  j.set("profile", m.profile.to_json());
  j.set("cublas_gflops", m.cublas_gflops ? json::Value(*m.cublas_gflops) : json::Value());
  return j;
}

int cmd_tune(const Args &a) {
  B200Runner::Options ro = runner_options(a);
  const GPU hw = b200_gpu(ro.dtype);
  const Problem prob = problem_of(a);
  B200Runner runner(ro);
  auto advisor = make_advisor(a.get("advisor", "rules"), a.get("kg", "knowledge/pass_graph.json"), a.get("llm-cmd", ""));
  TuneOptions o;
  o.budget = a.geti("budget", 30);
  o.seed = static_cast<uint64_t>(a.geti("seed", 0));
  o.log = [](const std::string &s) { std::puts(s.c_str()); };
  json::Value tr = tune_fanout(prob, hw, runner, *advisor, o, ro.fanout);
  const std::string out = a.get("out", "runs/trace_b200.json");
  const auto parent = std::filesystem::path(out).parent_path();
  if (!parent.empty()) std::filesystem::create_directories(parent);
  std::ofstream(out) << tr.dump(1);
  auto num = [&](const char *k) { return tr.at(k).is_null() ? std::string("n/a") : tr.at(k).dump(); };
  std::printf("\nsource=%s dtype=%s gpus=%d fanout=%d space=%s configs trials=%zu\n",
              tr.at("source").as_string().c_str(), pf_dtype_name(ro.dtype), ro.gpus, ro.fanout,
              num("space_size").c_str(), tr.at("trials").size());
  std::printf("baseline %s -> best %s GFLOP/s\ntrace -> %s\n", num("baseline_gflops").c_str(), num("best_gflops").c_str(),
              out.c_str());
  return 0;
}

int cmd_measure(const Args &a) {
  B200Runner::Options ro = runner_options(a);
  const GPU hw = b200_gpu(ro.dtype);
  Config c{a.geti("BM", 128), a.geti("BN", 256), a.geti("BK", 32), a.geti("TM", 4), a.geti("TN", 16), a.geti("PAD", 0)};
  B200Runner runner(ro);
  const Measurement m = runner.measure(c, problem_of(a), hw);
  json::Value j = measurement_json(m);
  j.set("cfg", c.to_json()).set("dtype", pf_dtype_name(ro.dtype)).set("gpus", ro.gpus);
  const auto unfused = runner.cublas_unfused_gflops();
  j.set("cublas_unfused_gflops", unfused ? json::Value(*unfused) : json::Value());
  std::puts(j.dump().c_str());
  return m.ok ? 0 : 4;
}

int cmd_gpus(const Args &a) {
  const GPU g = b200_gpu(parse_dtype(a.get("dtype", "bf16")));
  std::puts(g.to_json().dump().c_str());
  return 0;
}

}  // namespace

int main(int argc, char **argv) {
  if (argc < 2) {
    std::puts("usage: ptxforge-tune-b200 <tune|measure|gpus> [--key value ...]");
    return 64;
  }
  const std::string cmd = argv[1];
  try {
    Args a = Args::parse(argc, argv, 2);
    if (cmd == "tune") return cmd_tune(a);
    if (cmd == "measure") return cmd_measure(a);
    if (cmd == "gpus") return cmd_gpus(a);
    std::puts("usage: ptxforge-tune-b200 <tune|measure|gpus> [--key value ...]");
    return 64;
  } catch (const std::exception &e) {
    std::fprintf(stderr, "error: %s\n", e.what());
    return 1;
  }
}

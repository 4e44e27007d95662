// tune_fanout.hpp -- PTXForge's closed-loop search with trials fanned out over the GPUs of one box.
//
// ptxforge::tune (core/include/ptxforge/search.hpp:65-216) measures one config at a time.  tune_fanout()
// runs the same three phases -- the untuned baseline, the cost model's top picks, then advisor proposals /
// best-predicted neighbours of the incumbent -- but takes up to `width` candidates per round and hands
// them to a runner's measure_many(), which gates and times each on its own GPU(s) at the same time
// (B200Runner with Options::fanout = width).  The trace is the same schema-1 document tune() writes
// (search.hpp:186-214), trials in the order they were proposed, plus a top-level "fanout" object.
//
//   * width 1 is ptxforge::tune itself, so single-GPU traces are unchanged;
//   * the seeding phase proposes exactly tune()'s sequence (baseline, then the ranked list up to the seed
//     count) -- only the grouping into rounds differs;
//   * in the closed loop a round takes, in order: the advisor's valid unmeasured proposals for the
//     incumbent, then its unmeasured neighbours by predicted GFLOP/s, then the next best-predicted
//     configs of the whole space, until the round holds `width` configs or the budget is reached.
#pragma once

#include <algorithm>
#include <optional>
#include <set>
#include <string>
#include <tuple>
#include <vector>

#include "ptxforge/search.hpp"

namespace ptxforge {

template <class BatchRunner>
json::Value tune_fanout(const Problem &prob, const GPU &hw, BatchRunner &runner, Advisor &advisor,
                        const TuneOptions &opt, int width) {
  if (width <= 1) return tune(prob, hw, runner, advisor, opt);

  std::mt19937_64 rng(opt.seed);
  const std::vector<Config> space = enumerate_space(prob, hw);
  if (space.empty()) throw std::runtime_error("empty search space: problem size not divisible by any tile");
  std::map<Config, Analysis> model;
  for (const Config &c : space) model.emplace(c, analyze(c, prob, hw));
  auto analysis_of = [&](const Config &c) {
    auto it = model.find(c);
    return it != model.end() ? it->second : analyze(c, prob, hw);
  };
  auto predicted = [&](const Config &c) { return model.at(c).predicted_gflops; };
  std::vector<Config> ranked = space;
  std::stable_sort(ranked.begin(), ranked.end(),
                   [&](const Config &a, const Config &b) { return predicted(a) > predicted(b); });

  struct Done {
    Config cfg;
    std::optional<double> gflops;  // set when the trial passed
    Profile profile;
    std::vector<std::string> symptoms;
    double predicted;
    std::optional<double> cublas;
    json::Value json;
  };
  std::vector<Done> done;
  std::set<Config> measured;
  std::vector<HistoryEntry> history;
  int rounds = 0;
  auto hundredths = [](double x) { return std::round(x * 100.0) / 100.0; };

  struct Pick {
    Config cfg;
    std::string origin, why;
  };

  // Measure one round and append its trials in proposal order.
  auto measure_round = [&](const std::vector<Pick> &round) {
    std::vector<Config> cfgs;
    for (const Pick &p : round) cfgs.push_back(p.cfg);
    const std::vector<Measurement> ms = runner.measure_many(cfgs, prob, hw);
    ++rounds;
    for (size_t i = 0; i < round.size(); ++i) {
      const Pick &pk = round[i];
      const Measurement &m = ms[i];
      const Analysis an = analysis_of(pk.cfg);
      measured.insert(pk.cfg);
      Done d{pk.cfg, m.ok ? m.gflops : std::nullopt, m.profile, {}, an.predicted_gflops, m.cublas_gflops, {}};
      if (m.ok) d.symptoms = diagnose(pk.cfg, an, m.profile);

      json::Value j = json::Value::object();
      j.set("i", done.size()).set("cfg", pk.cfg.to_json()).set("origin", pk.origin).set("why", pk.why).set("ok", m.ok);
      j.set("error", m.ok ? json::Value() : json::Value(m.error));
      j.set("gflops", m.gflops ? json::Value(hundredths(*m.gflops)) : json::Value());
      j.set("ms", m.ms ? json::Value(std::round(*m.ms * 1e4) / 1e4) : json::Value());
      j.set("profile", m.profile.to_json());
      json::Value sym = json::Value::array();
      for (const auto &s : d.symptoms) sym.push_back(s);
      j.set("symptoms", sym);
      const json::Value full = an.to_json();
      json::Value modeled = json::Value::object();
      for (const char *k : {"ai", "ai_ideal", "roof_gflops", "memory_bound", "occupancy", "bank", "bank_degree",
                            "spill_regs", "predicted_gflops", "waves"})
        modeled.set(k, full.at(k));
      j.set("modeled", modeled);
      j.set("cublas_gflops", m.cublas_gflops ? json::Value(*m.cublas_gflops) : json::Value());
      d.json = j;
      history.push_back({pk.cfg, m.gflops ? std::optional<double>(hundredths(*m.gflops)) : std::nullopt});
      if (opt.log) {
        char head[200];
        std::snprintf(head, sizeof head, "[%3zu] %-22s %-14s ", done.size(), pk.cfg.short_name().c_str(),
                      pk.origin.c_str());
        std::string line = head;
        if (m.ok) {
          char g[48];
          std::snprintf(g, sizeof g, "%g GFLOP/s", hundredths(*m.gflops));
          line += g;
        } else {
          line += "FAILED: " + m.error.substr(0, 60);
        }
        opt.log(line);
      }
      done.push_back(std::move(d));
    }
  };

  auto incumbent = [&]() -> std::optional<size_t> {
    std::optional<size_t> best;
    for (size_t i = 0; i < done.size(); ++i)
      if (done[i].gflops && (!best || *done[i].gflops > *done[*best].gflops)) best = i;
    return best;
  };

  // Phase 1 -- baseline then the cost model's ranking, tune()'s sequence cut into rounds of `width`.
  const Config base_cfg = is_valid(kDefaultConfig, prob, hw)
                              ? kDefaultConfig
                              : *std::max_element(space.begin(), space.end(), [&](const Config &a, const Config &b) {
                                  return predicted(a) < predicted(b);
                                });
  const size_t n_seed = static_cast<size_t>(opt.seed_trials ? *opt.seed_trials : std::max(2, opt.budget / 4));
  std::vector<Pick> seeds{{base_cfg, "baseline", "untuned default"}};
  for (const Config &c : ranked) {
    if (seeds.size() >= std::max<size_t>(n_seed, 1)) break;
    if (c != base_cfg) seeds.push_back({c, "cost-model", "top predicted"});
  }
  for (size_t s = 0; s < seeds.size(); s += static_cast<size_t>(width))
    measure_round(std::vector<Pick>(seeds.begin() + s,
                                    seeds.begin() + std::min(seeds.size(), s + static_cast<size_t>(width))));

  // Phase 2 -- closed loop around the incumbent, `width` proposals per round.
  while (done.size() < static_cast<size_t>(opt.budget)) {
    const size_t room = std::min(static_cast<size_t>(width), static_cast<size_t>(opt.budget) - done.size());
    std::vector<Pick> round;
    std::set<Config> taken = measured;
    auto offer = [&](const Config &c, const std::string &origin, const std::string &why) {
      if (round.size() < room && !taken.count(c) && is_valid(c, prob, hw)) {
        taken.insert(c);
        round.push_back({c, origin, why});
      }
    };
    if (auto bi = incumbent()) {
      const Done &b = done[*bi];
      Context ctx{prob, hw, b.cfg, model.at(b.cfg), b.profile, b.symptoms, history, measured, rng};
      for (Proposal &p : advisor.propose(ctx)) offer(p.cfg, "advisor:" + advisor.name(), p.why);
      std::vector<Config> near = neighbors(b.cfg, prob, hw);
      std::stable_sort(near.begin(), near.end(), [&](const Config &x, const Config &y) {
        return predicted(x) > predicted(y);
      });
      for (const Config &n : near) offer(n, "neighbor", "best-predicted neighbor of incumbent");
    }
    for (const Config &c : ranked) offer(c, "cost-model", "next best predicted");
    if (round.empty()) break;
    measure_round(round);
  }

  // The trace: tune()'s schema-1 document.
  const auto bi = incumbent();
  const Done &base = done.front();
  std::vector<double> xs, ys;
  std::optional<double> cublas;
  for (const Done &d : done) {
    if (d.gflops) {
      xs.push_back(d.predicted);
      ys.push_back(*d.gflops);
    }
    if (!cublas && d.cublas) cublas = d.cublas;
  }
  const bool simulated = runner.source() == "simulated";
  json::Value out = json::Value::object();
  out.set("schema", 1).set("source", runner.source());
  out.set("warning", simulated ? json::Value("SIMULATED: numbers come from the analytic cost model plus noise, not "
                                             "a GPU. Do not quote them as results.")
                               : json::Value());
  out.set("created", iso_now());
  json::Value pj = json::Value::object();
  pj.set("M", prob.M).set("N", prob.N).set("K", prob.K).set("flops", prob.flops());
  out.set("problem", pj).set("gpu", hw.to_json()).set("advisor", advisor.name()).set("budget", opt.budget)
      .set("seed", opt.seed).set("space_size", space.size());
  out.set("baseline_gflops", base.gflops ? json::Value(hundredths(*base.gflops)) : json::Value());
  out.set("best_gflops", bi ? json::Value(hundredths(*done[*bi].gflops)) : json::Value());
  out.set("best_index", bi ? json::Value(*bi) : json::Value());
  out.set("speedup_vs_default", bi && base.gflops
                                    ? json::Value(std::round(*done[*bi].gflops / *base.gflops * 1000.0) / 1000.0)
                                    : json::Value());
  out.set("cublas_gflops", cublas ? json::Value(*cublas) : json::Value());
  out.set("pct_of_cublas",
          bi && cublas ? json::Value(std::round(100.0 * *done[*bi].gflops / *cublas * 10.0) / 10.0) : json::Value());
  const auto rho = spearman(xs, ys);
  out.set("model_spearman", rho ? json::Value(*rho) : json::Value());
  json::Value tj = json::Value::array();
  for (const Done &d : done) tj.push_back(d.json);
  out.set("trials", tj);
  json::Value st = json::Value::array();
  if (bi)
    for (const Stage &s : runner.stages(done[*bi].cfg, prob, hw)) {
      json::Value sj = json::Value::object();
      sj.set("name", s.name).set("lang", s.lang).set("text", s.text);
      st.push_back(sj);
    }
  out.set("stages", st);
  json::Value fo = json::Value::object();
  fo.set("width", width).set("rounds", rounds);
  out.set("fanout", fo);
  return out;
}

}  // namespace ptxforge

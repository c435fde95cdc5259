// Stage planner (host only): contiguous layer segments on distinct devices,
// chosen by an exact dynamic program.  Restates the cost model and search of
// AutoPlanner (dial-core/src/spm/planner.rs):
//   validate              planner.rs:576-741  (profile checks, same messages)
//   segment_cost          planner.rs:743-836  (memory, compute, hand-off, score)
//   initial/extend_cost   planner.rs:526-562  (the three objectives)
//   plan_with_algorithm   planner.rs:378-522  (DP over end layer x device set x last device)
// The search keeps, per state, the best cost and a back pointer instead of the
// reference's copied segment list; with the same visiting order and tie rules
// (lower score, then lower TTFT; at the end lower score, then fewer segments)
// it picks the same plan.
#include <cmath>
#include <cstring>
#include <vector>

#include "common.cuh"

namespace dial {
namespace {

constexpr double kMiB = 1024.0 * 1024.0;

double msum(const dial_layer_metric& m, int a, int b) {  // layers [a, b)
  if (!m.per_layer) return m.uniform * (double)(b - a);
  double s = 0.0;
  for (int i = a; i < b; ++i) s += m.per_layer[i];
  return s;
}
double mval(const dial_layer_metric& m, int i) { return m.per_layer ? m.per_layer[i] : m.uniform; }
bool bad(double v) { return !std::isfinite(v) || v < 0.0; }

dial_status check_metric(const dial_layer_metric& m, int L, const char* field, int dev) {
  if (!m.per_layer) {
    if (bad(m.uniform))
      return fail(DIAL_ERR_INVALID_ARG, "devices[%d].%s must be finite and non-negative, got %g", dev,
                  field, m.uniform);
    return DIAL_OK;
  }
  for (int i = 0; i < L; ++i)
    if (bad(m.per_layer[i]))
      return fail(DIAL_ERR_INVALID_ARG, "devices[%d].%s values must be finite and non-negative", dev, field);
  return DIAL_OK;
}

struct Cost {
  double ttft = 0, tpot = 0, tail_ttft = 0, tail_tpot = 0, energy = 0, score = 0;
};

struct Seg {
  int dev = -1, start = 0, end = 0;  // layers [start, end)
  double mem = 0, compute = 0, network = 0;
  Cost c;
};

struct State {
  bool set = false;
  Cost c;
  int prev_end = -1, prev_mask = 0, prev_last = -1;  // -1: first segment
  Seg seg;
  int nseg = 0;
};

struct Planner {
  const dial_plan_model& m;
  const dial_plan_objective& o;
  std::vector<const dial_plan_device*> dev;
  std::vector<int> dev_index;  // position in the caller's array
  double kv_mb_per_layer = 0;

  bool segment(int d, int a, int b, Seg& s) const {
    const dial_plan_device& D = *dev[d];
    const int L = m.num_layers;
    const bool first = a == 0, last = b == L;
    double mem = D.fixed_memory_mb + msum(D.layer_memory_mb, a, b) + kv_mb_per_layer * (b - a);
    double pre = msum(D.prefill_ms, a, b), dec = msum(D.decode_ms, a, b);
    double tpre = D.has_prefill_p95 ? msum(D.prefill_p95_ms, a, b) : pre;
    double tdec = D.has_decode_p95 ? msum(D.decode_p95_ms, a, b) : dec;
    if (first) {
      mem += m.embed_memory_mb;
      pre += m.embed_prefill_ms, tpre += m.embed_prefill_ms;
      dec += m.embed_decode_ms, tdec += m.embed_decode_ms;
    }
    if (last) {
      mem += m.head_memory_mb;
      pre += m.head_prefill_ms, tpre += m.head_prefill_ms;
      dec += m.head_decode_ms, tdec += m.head_decode_ms;
    }
    if (mem > D.usable_memory_mb) return false;
    // stage to stage: the master takes the prompt and the tokens, so it holds layer 0
    if (m.link_topology == DIAL_PLAN_LINKS_CHAIN && !first && D.role == DIAL_PLAN_MASTER) return false;
    s.dev = d, s.start = a, s.end = b, s.mem = mem;
    s.compute = pre + dec * o.output_tokens;
    Cost& c = s.c;
    c.ttft = pre + dec, c.tpot = dec, c.tail_ttft = tpre + tdec, c.tail_tpot = tdec;
    c.energy = msum(D.prefill_energy_mj, a, b) + msum(D.decode_energy_mj, a, b) * o.output_tokens;
    s.network = 0;
    const bool worker = D.role == DIAL_PLAN_WORKER;
    if (m.link_topology == DIAL_PLAN_LINKS_CHAIN) {
      // stage-to-stage hand-off: one hidden state per token into every segment
      // but the first (over the receiving device's link), and the token id back
      // from the last segment to the first
      const double in_pre = first ? 0.0 : (double)o.prompt_tokens * m.hidden_size * o.dtype_bytes;
      const double in_dec = first ? 0.0 : (double)m.hidden_size * o.dtype_bytes;
      const double out_tok = last && !first ? 4.0 : 0.0;
      if (worker && (in_dec > 0 || out_tok > 0)) {
        const double bw = D.bandwidth_mbps;
        const double tbw = D.bandwidth_p05_mbps >= 0 ? D.bandwidth_p05_mbps : bw;
        const double lat = D.rtt_ms + D.protocol_ms;
        const double tlat = (D.rtt_p95_ms >= 0 ? D.rtt_p95_ms : D.rtt_ms) +
                            (D.protocol_p95_ms >= 0 ? D.protocol_p95_ms : D.protocol_ms);
        const int hops = (in_dec > 0) + (out_tok > 0);
        const double pre_net = hops * lat + (in_pre + out_tok) * 8.0 / (bw * 1000.0);
        const double dec_net = hops * lat + (in_dec + out_tok) * 8.0 / (bw * 1000.0);
        const double tpre_net = hops * tlat + (in_pre + out_tok) * 8.0 / (tbw * 1000.0);
        const double tdec_net = hops * tlat + (in_dec + out_tok) * 8.0 / (tbw * 1000.0);
        s.network = pre_net + dec_net * o.output_tokens;
        c.ttft += pre_net + dec_net, c.tpot += dec_net;
        c.tail_ttft += tpre_net + tdec_net, c.tail_tpot += tdec_net;
      }
    } else if (worker) {
      const double bw = D.bandwidth_mbps;
      const double tbw = D.bandwidth_p05_mbps >= 0 ? D.bandwidth_p05_mbps : bw;
      const double trtt = D.rtt_p95_ms >= 0 ? D.rtt_p95_ms : D.rtt_ms;
      const double tproto = D.protocol_p95_ms >= 0 ? D.protocol_p95_ms : D.protocol_ms;
      // the segment's input comes in and its output goes back: 2 hidden states per token
      const double pre_bytes = 2.0 * o.prompt_tokens * m.hidden_size * (double)o.dtype_bytes;
      const double dec_bytes = 2.0 * m.hidden_size * (double)o.dtype_bytes;
      const double pre_net = D.rtt_ms + D.protocol_ms + pre_bytes * 8.0 / (bw * 1000.0);
      const double dec_net = D.rtt_ms + D.protocol_ms + dec_bytes * 8.0 / (bw * 1000.0);
      const double tpre_net = trtt + tproto + pre_bytes * 8.0 / (tbw * 1000.0);
      const double tdec_net = trtt + tproto + dec_bytes * 8.0 / (tbw * 1000.0);
      s.network = pre_net + dec_net * o.output_tokens;
      c.ttft += pre_net + dec_net, c.tpot += dec_net;
      c.tail_ttft += tpre_net + tdec_net, c.tail_tpot += tdec_net;
    }
    const double mean = o.ttft_weight * c.ttft + o.tpot_weight * c.tpot;
    const double tail = o.ttft_weight * c.tail_ttft + o.tpot_weight * c.tail_tpot;
    c.score = (1.0 - o.risk_weight) * mean + o.risk_weight * tail + o.energy_weight * c.energy +
              (worker ? o.remote_device_penalty : 0.0);
    return true;
  }

  static Cost initial(const Seg& s, int alg) {
    Cost c = s.c;
    if (alg == DIAL_PLAN_EDGESHARD_LATENCY) c.score = s.compute + s.network;
    else if (alg == DIAL_PLAN_EDGESHARD_THROUGHPUT) c.score = std::fmax(s.compute, s.network);
    return c;
  }

  static Cost extend(const Cost& cur, const Seg& s, int alg) {
    Cost c;
    c.ttft = cur.ttft + s.c.ttft, c.tpot = cur.tpot + s.c.tpot;
    c.tail_ttft = cur.tail_ttft + s.c.tail_ttft, c.tail_tpot = cur.tail_tpot + s.c.tail_tpot;
    c.energy = cur.energy + s.c.energy;
    if (alg == DIAL_PLAN_EDGESHARD_LATENCY) c.score = cur.score + s.compute + s.network;
    else if (alg == DIAL_PLAN_EDGESHARD_THROUGHPUT) c.score = std::fmax(std::fmax(cur.score, s.compute), s.network);
    else c.score = cur.score + s.c.score;
    return c;
  }
};

dial_status validate(const dial_plan_model& m, const dial_plan_objective& o,
                     const dial_plan_device* devices, int n, Planner& p) {
  if (m.num_layers <= 0) return fail(DIAL_ERR_INVALID_ARG, "model must have layers");
  if (m.link_topology != DIAL_PLAN_LINKS_STAR && m.link_topology != DIAL_PLAN_LINKS_CHAIN)
    return fail(DIAL_ERR_INVALID_ARG, "link_topology must be %d (star) or %d (chain)", DIAL_PLAN_LINKS_STAR,
                DIAL_PLAN_LINKS_CHAIN);
  if (o.prompt_tokens <= 0) return fail(DIAL_ERR_INVALID_ARG, "objective.prompt_tokens must be greater than zero");
  if (o.output_tokens <= 0) return fail(DIAL_ERR_INVALID_ARG, "objective.output_tokens must be greater than zero");
  if (o.dtype_bytes <= 0) return fail(DIAL_ERR_INVALID_ARG, "objective.dtype_bytes must be greater than zero");
  if (o.min_devices <= 0) return fail(DIAL_ERR_INVALID_ARG, "objective.min_devices must be greater than zero");
  if (m.num_attention_heads <= 0 || m.hidden_size % m.num_attention_heads)
    return fail(DIAL_ERR_INVALID_ARG, "model hidden_size %d is not divisible by num_attention_heads %d",
                m.hidden_size, m.num_attention_heads);
  const struct { const char* name; double v; } w[] = {
      {"ttft_weight", o.ttft_weight}, {"tpot_weight", o.tpot_weight}, {"risk_weight", o.risk_weight},
      {"energy_weight", o.energy_weight}, {"remote_device_penalty", o.remote_device_penalty}};
  for (const auto& x : w)
    if (bad(x.v)) return fail(DIAL_ERR_INVALID_ARG, "objective.%s must be finite and non-negative", x.name);
  if (o.risk_weight > 1.0) return fail(DIAL_ERR_INVALID_ARG, "objective.risk_weight must be between 0 and 1");
  if (o.ttft_weight == 0.0 && o.tpot_weight == 0.0 && o.energy_weight == 0.0)
    return fail(DIAL_ERR_INVALID_ARG, "at least one planning objective weight must be positive");
  for (const double v : {m.head_memory_mb, m.head_prefill_ms, m.head_decode_ms, m.embed_memory_mb,
                         m.embed_prefill_ms, m.embed_decode_ms})
    if (bad(v)) return fail(DIAL_ERR_INVALID_ARG, "head/embedding costs must be finite and non-negative");
  for (int i = 0; i < n; ++i)
    if (devices[i].enabled) {
      p.dev.push_back(&devices[i]);
      p.dev_index.push_back(i);
    }
  const int nd = (int)p.dev.size();
  if (nd == 0) return fail(DIAL_ERR_INVALID_ARG, "automatic planner profile has no enabled devices");
  if (nd > DIAL_PLAN_MAX_DEVICES)
    return fail(DIAL_ERR_INVALID_ARG, "automatic planner supports at most %d enabled devices", DIAL_PLAN_MAX_DEVICES);
  const int eff_max = o.max_devices > 0 && o.max_devices < nd ? o.max_devices : nd;
  if (o.min_devices > eff_max)
    return fail(DIAL_ERR_INVALID_ARG, "objective.min_devices (%d) exceeds the effective max_devices (%d)",
                o.min_devices, eff_max);
  int masters = 0;
  for (const auto* d : p.dev) masters += d->role == DIAL_PLAN_MASTER;
  if (masters != 1)
    return fail(DIAL_ERR_INVALID_ARG, "automatic planner requires exactly one enabled master, found %d", masters);
  const int L = m.num_layers;
  for (int k = 0; k < nd; ++k) {
    const dial_plan_device& d = *p.dev[k];
    const int id = p.dev_index[k];
    if (d.role != DIAL_PLAN_MASTER && d.role != DIAL_PLAN_WORKER)
      return fail(DIAL_ERR_INVALID_ARG, "devices[%d] has an unknown role", id);
    if (!std::isfinite(d.usable_memory_mb) || d.usable_memory_mb <= 0)
      return fail(DIAL_ERR_INVALID_ARG, "devices[%d] usable_memory_mb must be positive", id);
    if (bad(d.fixed_memory_mb) || d.fixed_memory_mb > d.usable_memory_mb)
      return fail(DIAL_ERR_INVALID_ARG, "devices[%d] has invalid fixed_memory_mb", id);
    dial_status s;
    if ((s = check_metric(d.layer_memory_mb, L, "layer_memory_mb", id)) != DIAL_OK) return s;
    if ((s = check_metric(d.prefill_ms, L, "prefill_ms", id)) != DIAL_OK) return s;
    if ((s = check_metric(d.decode_ms, L, "decode_ms", id)) != DIAL_OK) return s;
    if ((s = check_metric(d.prefill_energy_mj, L, "prefill_energy_mj", id)) != DIAL_OK) return s;
    if ((s = check_metric(d.decode_energy_mj, L, "decode_energy_mj", id)) != DIAL_OK) return s;
    const struct { int has; const dial_layer_metric* tail; const dial_layer_metric* mean; const char* tn;
                   const char* mn; } tails[] = {
        {d.has_prefill_p95, &d.prefill_p95_ms, &d.prefill_ms, "prefill_p95_ms", "prefill_ms"},
        {d.has_decode_p95, &d.decode_p95_ms, &d.decode_ms, "decode_p95_ms", "decode_ms"}};
    for (const auto& t : tails) {
      if (!t.has) continue;
      if ((s = check_metric(*t.tail, L, t.tn, id)) != DIAL_OK) return s;
      for (int i = 0; i < L; ++i)
        if (mval(*t.tail, i) < mval(*t.mean, i))
          return fail(DIAL_ERR_INVALID_ARG,
                      "devices[%d].%s at layer %d (%g) must be no smaller than devices[%d].%s (%g)", id,
                      t.tn, i, mval(*t.tail, i), id, t.mn, mval(*t.mean, i));
    }
    if (d.role == DIAL_PLAN_WORKER) {
      if (!std::isfinite(d.bandwidth_mbps) || d.bandwidth_mbps <= 0)
        return fail(DIAL_ERR_INVALID_ARG, "worker %d requires a positive bandwidth_mbps", id);
      if (bad(d.rtt_ms) || bad(d.protocol_ms))
        return fail(DIAL_ERR_INVALID_ARG, "worker %d has invalid network timings", id);
      const double trtt = d.rtt_p95_ms >= 0 ? d.rtt_p95_ms : d.rtt_ms;
      const double tproto = d.protocol_p95_ms >= 0 ? d.protocol_p95_ms : d.protocol_ms;
      const double tbw = d.bandwidth_p05_mbps >= 0 ? d.bandwidth_p05_mbps : d.bandwidth_mbps;
      if (!std::isfinite(trtt) || trtt < d.rtt_ms || !std::isfinite(tproto) || tproto < d.protocol_ms)
        return fail(DIAL_ERR_INVALID_ARG,
                    "worker %d tail network latencies must be finite and no smaller than their mean values", id);
      if (!std::isfinite(tbw) || tbw <= 0 || tbw > d.bandwidth_mbps)
        return fail(DIAL_ERR_INVALID_ARG,
                    "worker %d bandwidth_p05_mbps must be positive and no greater than bandwidth_mbps", id);
    }
  }
  const int head_dim = m.hidden_size / m.num_attention_heads;
  const int kv_ctx = o.kv_context_tokens == 0
                         ? m.max_seq_len
                         : (o.kv_context_tokens < m.max_seq_len ? o.kv_context_tokens : m.max_seq_len);
  p.kv_mb_per_layer = 2.0 * m.num_key_value_heads * head_dim * (double)kv_ctx * o.dtype_bytes / kMiB;
  return DIAL_OK;
}

}  // namespace
}  // namespace dial

using namespace dial;

extern "C" dial_status dial_plan_stages(const dial_plan_model* model, const dial_plan_objective* objective,
                                        const dial_plan_device* devices, int n_devices, int algorithm,
                                        dial_plan_result* out) {
  clear_error();
  if (!model || !objective || !devices || !out || n_devices <= 0)
    return fail(DIAL_ERR_INVALID_ARG, "null pointer or no devices");
  if (algorithm < DIAL_PLAN_DIAL || algorithm > DIAL_PLAN_EDGESHARD_THROUGHPUT)
    return fail(DIAL_ERR_INVALID_ARG, "unknown planner algorithm %d", algorithm);
  Planner p{*model, *objective, {}, {}, 0.0};
  dial_status s = validate(*model, *objective, devices, n_devices, p);
  if (s != DIAL_OK) return s;
  const int L = model->num_layers, D = (int)p.dev.size(), M = 1 << D;
  const int max_dev = objective->max_devices > 0 && objective->max_devices < D ? objective->max_devices : D;
  // dp[end][mask][last], end in 0..L
  std::vector<State> dp((size_t)(L + 1) * M * D);
  auto at = [&](int end, int mask, int last) -> State& { return dp[((size_t)end * M + mask) * D + last]; };
  int64_t states = 0, feasible = 0, rejected = 0;
  Seg seg;
  for (int d = 0; d < D; ++d)
    for (int end = 1; end <= L; ++end) {
      if (!p.segment(d, 0, end, seg)) {
        ++rejected;
        continue;
      }
      ++feasible;
      State& st = at(end, 1 << d, d);
      st.set = true, st.c = Planner::initial(seg, algorithm), st.seg = seg, st.nseg = 1;
    }
  for (int end = 1; end < L; ++end)
    for (int mask = 1; mask < M; ++mask) {
      if (__builtin_popcount(mask) >= max_dev) continue;
      for (int last = 0; last < D; ++last) {
        const State& cur = at(end, mask, last);
        if (!cur.set) continue;
        ++states;
        for (int nxt = 0; nxt < D; ++nxt) {
          if (mask & (1 << nxt)) continue;
          for (int ne = end + 1; ne <= L; ++ne) {
            if (!p.segment(nxt, end, ne, seg)) {
              ++rejected;
              continue;
            }
            ++feasible;
            const Cost c = Planner::extend(cur.c, seg, algorithm);
            State& slot = at(ne, mask | (1 << nxt), nxt);
            if (!slot.set || c.score < slot.c.score || (c.score == slot.c.score && c.ttft < slot.c.ttft)) {
              slot.set = true, slot.c = c, slot.seg = seg, slot.nseg = cur.nseg + 1;
              slot.prev_end = end, slot.prev_mask = mask, slot.prev_last = last;
            }
          }
        }
      }
    }
  const State* best = nullptr;
  for (int mask = 1; mask < M; ++mask) {
    const int k = __builtin_popcount(mask);
    if (k < objective->min_devices || k > max_dev) continue;
    for (int last = 0; last < D; ++last) {
      const State& c = at(L, mask, last);
      if (!c.set) continue;
      if (!best || c.c.score < best->c.score || (c.c.score == best->c.score && c.nseg < best->nseg)) best = &c;
    }
  }
  if (!best)
    return fail(DIAL_ERR_SHAPE,
                "automatic planner found no feasible placement for %d layers; check device memory profiles", L);
  std::memset(out, 0, sizeof(*out));
  out->n_segments = best->nseg;
  const State* st = best;
  for (int i = best->nseg - 1; i >= 0; --i) {
    dial_plan_segment& o = out->segments[i];
    o.device = p.dev_index[st->seg.dev];
    o.start_layer = st->seg.start;
    o.end_layer = st->seg.end - 1;
    o.memory_mb = st->seg.mem;
    o.ttft_ms = st->seg.c.ttft, o.tpot_ms = st->seg.c.tpot;
    o.tail_ttft_ms = st->seg.c.tail_ttft, o.tail_tpot_ms = st->seg.c.tail_tpot;
    if (i > 0) st = &at(st->prev_end, st->prev_mask, st->prev_last);
  }
  out->ttft_ms = best->c.ttft, out->tpot_ms = best->c.tpot;
  out->tail_ttft_ms = best->c.tail_ttft, out->tail_tpot_ms = best->c.tail_tpot;
  out->request_energy_mj = best->c.energy, out->score = best->c.score;
  out->states_considered = states, out->feasible_transitions = feasible, out->rejected_for_memory = rejected;
  return DIAL_OK;
}

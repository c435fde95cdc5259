"""Stage planner (dial_plan_stages) on the CPU.

The first group restates the reference's own planner tests
(dial-core/src/spm/planner.rs:953-1270) with the same profiles and expected
plans; the rest pins the B200 pipeline use (head weighting, brute force).
"""
import itertools

import pytest

from dial_cuda import DialError
from dial_cuda import planner as P


def config(layers):  # planner.rs:958-973
    return P.PlannerModel(num_layers=layers, hidden_size=4096, num_attention_heads=32,
                          num_key_value_heads=8, max_seq_len=1024)


def device(name, role, speed, memory):  # planner.rs:975-1000
    worker = role == P.WORKER
    return P.PlannerDevice(name=name, role=role, usable_memory_mb=memory, fixed_memory_mb=100.0,
                           layer_memory_mb=100.0, prefill_ms=speed, decode_ms=speed,
                           rtt_ms=0.2 if worker else 0.0,
                           bandwidth_mbps=1000.0 if worker else None)


def objective(**kw):  # planner.rs:1002-1016
    o = P.PlannerObjective(prompt_tokens=128, output_tokens=32, dtype_bytes=2, kv_context_tokens=128,
                           ttft_weight=0.6, tpot_weight=0.4)
    for k, v in kw.items():
        setattr(o, k, v)
    return o


def test_selects_only_fast_orin_when_it_can_hold_every_layer():
    r = P.plan_stages(config(8), objective(), [
        device("master", P.MASTER, 20.0, 5000.0), device("rk1", P.WORKER, 20.0, 5000.0),
        device("rk2", P.WORKER, 20.0, 5000.0), device("orin", P.WORKER, 1.0, 5000.0)])
    assert r["selected_device_count"] == 1
    s = r["segments"][0]
    assert (s["device"], s["start_layer"], s["end_layer"]) == ("orin", 0, 7)


def test_uses_optional_rk_workers_when_orin_cannot_hold_every_layer():
    r = P.plan_stages(config(8), objective(), [
        device("master", P.MASTER, 30.0, 250.0), device("rk1", P.WORKER, 10.0, 450.0),
        device("rk2", P.WORKER, 11.0, 450.0), device("orin", P.WORKER, 1.0, 450.0)])
    assert r["selected_device_count"] == 3
    assert sum(s["num_layers"] for s in r["segments"]) == 8
    assert any(s["device"] == "orin" for s in r["segments"])
    assert sum(s["device"].startswith("rk") for s in r["segments"]) == 2


def test_max_devices_is_respected_without_requiring_all_devices():
    r = P.plan_stages(config(8), objective(max_devices=2), [
        device("master", P.MASTER, 20.0, 5000.0), device("rk1", P.WORKER, 10.0, 5000.0),
        device("rk2", P.WORKER, 10.0, 5000.0), device("orin", P.WORKER, 1.0, 5000.0)])
    assert r["selected_device_count"] == 1


def test_min_devices_supports_the_no_subset_ablation():
    r = P.plan_stages(config(8), objective(min_devices=4, max_devices=4), [
        device("master", P.MASTER, 1.0, 10_000.0), device("rk1", P.WORKER, 1.0, 10_000.0),
        device("rk2", P.WORKER, 1.0, 10_000.0), device("orin", P.WORKER, 1.0, 10_000.0)])
    assert r["selected_device_count"] == 4
    assert all(s["num_layers"] > 0 for s in r["segments"])


def test_risk_weight_avoids_a_fast_but_unstable_worker():
    master = device("master", P.MASTER, 2.0, 10_000.0)
    unstable = device("unstable", P.WORKER, 1.0, 10_000.0)
    unstable.rtt_ms = 0.0
    unstable.bandwidth_mbps = 1_000_000.0
    unstable.prefill_p95_ms = 10.0
    unstable.decode_p95_ms = 10.0
    mean = P.plan_stages(config(8), objective(), [master, unstable])
    assert mean["segments"][0]["device"] == "unstable"
    robust = P.plan_stages(config(8), objective(risk_weight=1.0), [master, unstable])
    assert robust["segments"][0]["device"] == "master"
    assert robust["cost"]["tail_ttft_ms"] < mean["cost"]["tail_ttft_ms"]


def test_rejects_a_tail_profile_below_its_mean():
    worker = device("worker", P.WORKER, 2.0, 10_000.0)
    worker.prefill_p95_ms = 1.0
    with pytest.raises(DialError, match="must be no smaller than"):
        P.plan_stages(config(8), objective(), [device("master", P.MASTER, 2.0, 10_000.0), worker])


def test_edgeshard_latency_prefers_one_fast_segment_for_a_single_request():
    r = P.plan_stages(config(8), objective(), [device("master", P.MASTER, 1.0, 10_000.0),
                                               device("worker", P.WORKER, 2.0, 10_000.0)],
                      P.EDGESHARD_LATENCY)
    assert r["selected_device_count"] == 1
    assert r["segments"][0]["device"] == "master"
    assert r["score_definition"] == "estimated_end_to_end_request_latency_ms"


def test_edgeshard_throughput_balances_the_pipeline_bottleneck():
    worker = device("worker", P.WORKER, 1.0, 10_000.0)
    worker.rtt_ms = 0.0
    worker.bandwidth_mbps = 1_000_000.0
    r = P.plan_stages(config(8), objective(), [device("master", P.MASTER, 1.0, 10_000.0), worker],
                      P.EDGESHARD_THROUGHPUT)
    assert r["selected_device_count"] == 2
    assert sum(s["num_layers"] for s in r["segments"]) == 8
    assert r["cost"]["score"] < 8.0 * 33.0


def test_rejects_a_profile_without_exactly_one_master():
    with pytest.raises(DialError, match="exactly one enabled master"):
        P.plan_stages(config(8), objective(), [device("a", P.WORKER, 1.0, 10_000.0),
                                               device("b", P.WORKER, 1.0, 10_000.0)])


def test_no_feasible_placement_reports_shape_error():
    with pytest.raises(DialError, match="no feasible placement"):
        P.plan_stages(config(8), objective(), [device("master", P.MASTER, 1.0, 300.0)])


# ---------------------------------------------------------------- B200 pipeline use
def _brute_bottleneck(costs, k):
    """Min over all splits of the layer-cost list into k contiguous parts of the max part."""
    n = len(costs)
    best = None
    for cuts in itertools.combinations(range(1, n), k - 1):
        b = (0,) + cuts + (n,)
        m = max(sum(costs[b[i]:b[i + 1]]) for i in range(k))
        best = m if best is None else min(best, m)
    return best


@pytest.mark.parametrize("layers,gpus,head", [(36, 2, 3.2), (36, 4, 3.2), (12, 3, 2.0), (9, 4, 0.0)])
def test_local_gpu_plan_minimises_the_bottleneck(layers, gpus, head):
    ranges = P.local_gpu_plan(layers, gpus, head_layers=head, layer_decode_ms=1.0,
                              link_latency_ms=0.0)
    assert len(ranges) == gpus
    assert ranges[0].start == 0 and ranges[-1].stop == layers
    assert all(a.stop == b.start for a, b in zip(ranges, ranges[1:]))
    costs = [1.0] * layers
    costs[-1] += head  # the head rides with the last layer's stage
    got = max(sum(costs[r.start:r.stop]) for r in ranges)
    assert got == pytest.approx(_brute_bottleneck(costs, gpus))


def test_local_gpu_plan_even_without_head_weight():
    assert [len(r) for r in P.local_gpu_plan(36, 4, link_latency_ms=0.0)] == [9, 9, 9, 9]
    assert sorted(len(r) for r in P.local_gpu_plan(36, 8, link_latency_ms=0.0)) == [4, 4, 4, 4, 5, 5, 5, 5]


# ---------------------------------------------------------------- stage-to-stage links
def _chain_devices(n, rtt, proto=0.0, mbps=8000.0):
    return [P.PlannerDevice(name=f"gpu{i}", role=P.MASTER if i == 0 else P.WORKER,
                            usable_memory_mb=250.0 if n > 1 else 5000.0, fixed_memory_mb=0.0,
                            layer_memory_mb=100.0, prefill_ms=1.0, decode_ms=1.0,
                            rtt_ms=rtt if i else 0.0, protocol_ms=proto if i else 0.0,
                            bandwidth_mbps=mbps if i else None)
            for i in range(n)]


def test_chain_links_charge_one_hidden_state_into_each_later_stage():
    """Four 2-layer stages (memory forces the split): stage s > 0 pays one
    incoming hand-off per token (rtt + protocol + H * dtype bytes over its
    link), the last stage also the 4-byte token back; stage 0 (the master,
    which holds layer 0 under the chain model) pays nothing."""
    m = config(8)
    m.link_topology = P.LINKS_CHAIN
    rtt, proto, mbps = 0.5, 0.25, 8000.0
    r = P.plan_stages(m, objective(min_devices=4, max_devices=4), _chain_devices(4, rtt, proto, mbps))
    segs = sorted(r["segments"], key=lambda s: s["start_layer"])
    assert [s["num_layers"] for s in segs] == [2, 2, 2, 2]
    hop = rtt + proto
    hidden = 4096 * 2 * 8.0 / (mbps * 1000.0)
    tok = 4 * 8.0 / (mbps * 1000.0)
    want = [2.0, 2.0 + hop + hidden, 2.0 + hop + hidden, 2.0 + 2 * hop + hidden + tok]
    assert [s["estimated_tpot_ms"] for s in segs] == pytest.approx(want, rel=1e-12)
    assert segs[0]["device"] == "gpu0"


def test_star_links_keep_the_reference_cost():
    """The default (star): a worker segment pays 2 hidden states per token plus
    one rtt + protocol per direction-pair, as planner.rs:787-805."""
    m = config(8)
    rtt, proto, mbps = 0.5, 0.25, 8000.0
    r = P.plan_stages(m, objective(min_devices=4, max_devices=4), _chain_devices(4, rtt, proto, mbps))
    segs = sorted(r["segments"], key=lambda s: s["start_layer"])
    star = 2.0 + rtt + proto + 2 * 4096 * 2 * 8.0 / (mbps * 1000.0)
    by_dev = {s["device"]: s["estimated_tpot_ms"] for s in segs}
    assert by_dev.pop("gpu0") == pytest.approx(2.0)  # the master pays no link
    assert sorted(by_dev.values()) == pytest.approx([star] * 3, rel=1e-12)


def test_slow_chain_links_favour_fewer_stages():
    """With 3 ms per hop the planner keeps all 8 layers on one GPU when it can
    (4 stages would add 3 hops + the token's return per token)."""
    m = config(8)
    m.link_topology = P.LINKS_CHAIN
    devs = _chain_devices(4, 3.0)
    for d in devs:
        d.usable_memory_mb = 5000.0
    r = P.plan_stages(m, objective(), devs)
    assert r["selected_device_count"] == 1


def test_rejects_an_unknown_link_topology():
    m = config(8)
    m.link_topology = 7
    with pytest.raises(DialError, match="link_topology"):
        P.plan_stages(m, objective(), _chain_devices(2, 0.1))

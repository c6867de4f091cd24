"""The coordinator's scheduling decisions in the runtime library (csrc/runtime/scheduler.cpp) against a
plain-Python statement of the reference rules (coordinator/src/state.rs:63-225, routes.rs:244-263) on
randomised states."""
import datetime as dt
import math
import random

from distrain_b200 import protocol as P

T0 = dt.datetime(2026, 1, 1, tzinfo=dt.timezone.utc)


def _oracle_accept(acc, push, decay, max_st):
    st = max(acc.checkpoint_version - push.checkpoint_version, 0)
    if st > max_st:
        return False, f"Too stale: {st} > {max_st}", None
    for c in acc.contributions:
        if c.node_id == push.node_id and c.seq_num >= push.seq_num:
            return False, f"Duplicate: existing seq_num {c.seq_num} >= {push.seq_num}", None
    return True, None, push.tokens_processed * decay ** st


def _oracle_trigger(acc, min_override, cs, now):
    n = len(acc.contributions)
    if n == 0:
        return False
    active = len(cs.heartbeats)
    req = min_override if min_override > 0 else (1 if active <= 1 else max(active // 2, 2))
    if n < req:
        return False
    contributing = {c.node_id for c in acc.contributions}
    if active > 0 and sum(1 for nid in cs.heartbeats if nid in contributing) >= active:
        return True
    elapsed = float(int(max((now - acc.first_contribution_at).total_seconds(), 0.0)))
    times = sorted(t for nid, p in cs.node_profiles.items() if nid in cs.heartbeats
                   for t in [p.expected_round_time if p.expected_round_time is not None else p.round_time_secs]
                   if t is not None)
    if not times:
        patience = 60.0
    else:
        med = times[len(times) // 2]
        cl = [t for t in times if t <= med * 3.0]
        patience = min(max((cl[-1] if cl else med) * 1.2, 30.0), 300.0)
    return elapsed >= patience


def test_accept_push_matches_rules():
    rnd = random.Random(0)
    for trial in range(400):
        acc = P.AccumulatorState(checkpoint_version=rnd.randint(0, 20))
        for i in range(rnd.randint(0, 6)):
            acc.contributions.append(P.ContributionMeta(node_id=f"n{rnd.randint(0, 4)}", seq_num=rnd.randint(0, 9),
                                                        weight=1.0, checkpoint_version=0, inner_steps=1,
                                                        tokens_processed=1, delta_key="k",
                                                        received_at=T0))
        push = P.DeltaPush(node_id=f"n{rnd.randint(0, 4)}", seq_num=rnd.randint(0, 12),
                           checkpoint_version=rnd.randint(0, 22), inner_steps=5, delta_key="d",
                           training_loss=1.0, tokens_processed=rnd.randint(1, 10 ** 6), training_time_secs=1.0)
        decay, max_st = rnd.choice([0.9, 0.5, 1.0]), rnd.randint(0, 12)
        want_ok, want_reason, want_w = _oracle_accept(acc, push, decay, max_st)
        before = len(acc.contributions)
        ok, reason = P.apply_delta_push(acc, push, decay, max_st)
        assert ok == want_ok and reason == want_reason, (trial, ok, reason, want_reason)
        if ok:
            mine = [c for c in acc.contributions if c.node_id == push.node_id]
            assert len(mine) == 1 and abs(mine[0].weight - want_w) <= 1e-9 * max(1.0, want_w)
        else:
            assert len(acc.contributions) == before


def test_trigger_matches_rules():
    rnd = random.Random(1)
    t0 = dt.datetime(2026, 1, 1, tzinfo=dt.timezone.utc)
    for trial in range(600):
        acc = P.AccumulatorState()
        cs = P.CoordinatorPersistentState()
        nodes = [f"n{i}" for i in range(rnd.randint(1, 9))]
        for nid in nodes:
            if rnd.random() < 0.8:
                cs.heartbeats[nid] = 1
            prof = P.NodeProfile()
            r = rnd.random()
            if r < 0.3:
                prof.expected_round_time = rnd.uniform(1, 400)
            elif r < 0.6:
                prof.round_time_secs = rnd.uniform(1, 400)
            cs.node_profiles[nid] = prof
        for nid in rnd.sample(nodes, rnd.randint(0, len(nodes))):
            acc.contributions.append(P.ContributionMeta(node_id=nid, seq_num=1, weight=1.0, checkpoint_version=0,
                                                        inner_steps=1, tokens_processed=1, delta_key="k", received_at=T0))
        acc.first_contribution_at = t0
        now = t0 + dt.timedelta(seconds=rnd.uniform(0, 400))
        mo = rnd.choice([0, 0, 1, 3])
        assert P.should_checkpoint(acc, mo, cs, now) == _oracle_trigger(acc, mo, cs, now), trial


def test_round_time_ema():
    cs = P.CoordinatorPersistentState()
    cs.node_profiles["a"] = P.NodeProfile()
    P.update_round_time(cs, "a", 1000)       # first push: no interval yet
    assert cs.node_profiles["a"].round_time_secs is None
    P.update_round_time(cs, "a", 1100)       # 100 s
    assert cs.node_profiles["a"].round_time_secs == 100.0
    P.update_round_time(cs, "a", 1105)       # 5 s: ignored
    assert cs.node_profiles["a"].round_time_secs == 100.0
    P.update_round_time(cs, "a", 1155)       # 50 s: 0.3 * 100 + 0.7 * 50
    assert math.isclose(cs.node_profiles["a"].round_time_secs, 65.0)
    assert cs.node_profiles["a"].last_push_time == 1155

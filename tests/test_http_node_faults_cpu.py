"""HTTP node against network faults on the push: a push that fails in transit is retried with backoff and
accepted; a push whose reply is lost (the coordinator took it) is retried, meets the coordinator's dedup
by sequence number, and counts as delivered."""
import pytest

from distrain_b200.utils.data import SyntheticTokens

from test_node_resume_cpu import CFG, _node, _service


@pytest.mark.timeout(300)
def test_push_retries_and_lost_reply(tmp_path):
    store, svc, url = _service(tmp_path, min_contributions=10)  # no merges: the pushes stay in the accumulator
    try:
        n = _node(url, store, SyntheticTokens(CFG.vocab_size, 2, 17, seed=1).next_batch, None, node_id="flaky")
        n.register()
        real = n.client.push_delta
        calls = []

        def flaky(push):
            calls.append(push.seq_num)
            if push.seq_num == 1 and calls.count(1) == 1:
                raise ConnectionError("injected: connection reset before the request arrived")
            if push.seq_num == 2 and calls.count(2) == 1:
                real(push)  # the coordinator takes it ...
                raise ConnectionError("injected: ... and the reply is lost")
            return real(push)
        n.client.push_delta = flaky
        n.run(11)  # pushes after steps 5 and 10
        assert not n.errors, n.errors
        assert [(p["seq"], p["accepted"]) for p in n.pushes] == [(1, True), (2, True)]
        assert calls == [1, 1, 2, 2]
        assert any(p["reason"] and "Duplicate" in p["reason"] for p in n.pushes)  # seq 2's retry met the dedup
        assert [c.seq_num for c in svc.acc.state.contributions if c.node_id == "flaky"] == [2]
    finally:
        svc.stop()

"""Monitoring assets agree with the exported metrics: every distrain_* series that the alert rules and the
dashboard query is one the coordinator exports; the in-box /metrics server answers."""
import json
import os
import re
import urllib.request

import yaml

from distrain_b200.coordinator.metrics import Metrics, MetricsServer

MON = os.path.join(os.path.dirname(__file__), "..", "distrain_b200", "coordinator", "monitoring")


def _exported():
    m = Metrics()
    return set(re.findall(r"^(distrain_\w+) ", m.render(), re.M))


def test_alerts_and_dashboard_reference_exported_series():
    names = _exported()
    rules = yaml.safe_load(open(os.path.join(MON, "alerts.yml")))["groups"][0]["rules"]
    assert {r["alert"] for r in rules} == {"AccumulatorStall", "HighRejectionRate", "AggregationFailures",
                                           "NoActiveNodes"}
    exprs = [r["expr"] for r in rules]
    dash = json.load(open(os.path.join(MON, "grafana", "distrain_b200.json")))
    assert len(dash["panels"]) == 10
    exprs += [t["expr"] for p in dash["panels"] for t in p["targets"]]
    used = set(re.findall(r"distrain_\w+", " ".join(exprs)))
    assert used and used <= names, used - names
    prom = yaml.safe_load(open(os.path.join(MON, "prometheus.yml")))
    assert prom["rule_files"] == ["alerts.yml"]


def test_inbox_metrics_server():
    m = Metrics()
    m.checkpoint_version = 7
    srv = MetricsServer(m, host="127.0.0.1", port=0)
    try:
        body = urllib.request.urlopen(f"http://127.0.0.1:{srv.port}/metrics", timeout=10).read().decode()
        assert "distrain_checkpoint_version 7" in body
        assert urllib.request.urlopen(f"http://127.0.0.1:{srv.port}/health", timeout=10).read() == b"ok"
    finally:
        srv.stop()

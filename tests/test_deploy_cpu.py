"""Deployment surface: container image, entrypoints, compose stack, monitoring wiring, task runner,
project metadata and CI, checked without Docker or a GPU:

* every file the Dockerfile copies and every path the compose stack mounts exists;
* Prometheus scrapes the compose services on the ports they serve, and loads the alert rules;
* each entrypoint, run with DT_DRY_RUN=1, prints commands that the CLI parser accepts; the node
  entrypoint writes a node.toml that NodeConfig reads back with the environment's values, and the start
  command resolves its coordinator, device, batch and push interval from it;
* ``bootstrap --if-absent`` creates checkpoint v0 once; a missing --store means the R2_* environment;
* every Makefile target expands (make -n) and the CI workflow runs existing targets;
* the console script and the package data in pyproject.toml resolve."""
import glob
import importlib
import os
import re
import shlex
import shutil
import subprocess
import tomllib

import pytest
import yaml

from distrain_b200 import cli
from distrain_b200.config import NodeConfig

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DEPLOY = os.path.join(ROOT, "deploy")


def _dry(script, env):
    e = {"PATH": os.environ["PATH"], "DT_DRY_RUN": "1", "PYTHON": "python"}
    e.update(env)
    r = subprocess.run(["bash", os.path.join(DEPLOY, script)], env=e, capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    return r.stdout


def _cli_args(line):
    """The distrain_b200 argument list of a printed `python -m distrain_b200 ...` command line."""
    toks = shlex.split(line)
    return toks[toks.index("distrain_b200") + 1:]


def test_dockerfile_copies_existing_paths():
    text = open(os.path.join(DEPLOY, "Dockerfile")).read()
    copies = re.findall(r"^COPY (.+)$", text, re.M)
    assert copies
    for line in copies:
        for src in line.split()[:-1]:
            assert os.path.exists(os.path.join(ROOT, src)), src
    for ep in ("entrypoint-coordinator.sh", "entrypoint-node.sh", "entrypoint-box.sh"):
        assert os.access(os.path.join(DEPLOY, ep), os.X_OK), ep


def test_compose_mounts_and_monitoring_wiring():
    c = yaml.safe_load(open(os.path.join(DEPLOY, "compose.yml")))
    svcs = c["services"]
    for name, s in svcs.items():
        for v in s.get("volumes", []):
            src = v.split(":")[0]
            if src.startswith("."):
                assert os.path.exists(os.path.normpath(os.path.join(DEPLOY, src))), (name, src)
        b = s.get("build")
        if b:
            ctx = os.path.normpath(os.path.join(DEPLOY, b["context"]))
            assert os.path.exists(os.path.join(ctx, b["dockerfile"]))
    prom = yaml.safe_load(open(os.path.join(DEPLOY, "prometheus.yml")))
    assert prom["rule_files"] == ["alerts.yml"]
    targets = {j["job_name"]: j["static_configs"][0]["targets"][0] for j in prom["scrape_configs"]}
    host, port = targets["distrain-coordinator"].split(":")
    assert host in svcs and svcs[host]["environment"]["PORT"] == port
    host, port = targets["distrain-inbox"].split(":")
    assert host in svcs and svcs[host]["environment"]["METRICS_PORT"] == port
    # the host-local scrape config has the same jobs
    local = yaml.safe_load(open(os.path.join(ROOT, "distrain_b200/coordinator/monitoring/prometheus.yml")))
    assert {j["job_name"] for j in local["scrape_configs"]} == set(targets)
    alerts = yaml.safe_load(open(os.path.join(ROOT, "distrain_b200/coordinator/monitoring/alerts.yml")))
    assert sum(len(g["rules"]) for g in alerts["groups"]) == 4


def test_node_entrypoint_writes_a_node_config_the_start_command_reads(tmp_path):
    cfg = tmp_path / "node.toml"
    out = _dry("entrypoint-node.sh", {"NODE_CONFIG": str(cfg), "COORDINATOR_URL": "http://coord:8123",
                                      "S3_ENDPOINT": "http://store:9000", "S3_BUCKET": "bkt", "GPU_DEVICE": "3",
                                      "BATCH_SIZE": "6", "SEQ_LEN": "1024", "MIN_INNER_STEPS": "25",
                                      "CACHE_DIR": str(tmp_path / "cache")})
    nc = NodeConfig.load_toml(str(cfg))
    assert (nc.coordinator_url, nc.gpu_device, nc.force_batch_size, nc.seq_len) == ("http://coord:8123", 3, 6, 1024)
    assert (nc.storage.endpoint, nc.storage.bucket) == ("http://store:9000", "bkt")
    cmd = [ln for ln in out.splitlines() if "distrain_b200" in ln][-1]
    args = cli.build_parser().parse_args(_cli_args(cmd))
    assert args.fn is cli.cmd_start
    cli._apply_node_config(args)
    assert (args.coordinator_url, args.device, args.batch_size, args.seq_len, args.h_mini) == \
        ("http://coord:8123", "cuda:3", 6, 1024, 25)
    assert args.storage_cfg.endpoint == "http://store:9000"


def test_coordinator_entrypoint_commands_parse():
    out = _dry("entrypoint-coordinator.sh", {"PRESET": "small", "PORT": "8111", "R2_ENDPOINT": "http://s:9000"})
    lines = [ln for ln in out.splitlines() if "distrain_b200" in ln]
    assert len(lines) == 2
    boot = cli.build_parser().parse_args(_cli_args(lines[0]))
    assert boot.fn is cli.cmd_bootstrap and boot.if_absent and boot.preset == "small" and boot.store is None
    coord = cli.build_parser().parse_args(_cli_args(lines[1]))
    assert coord.fn is cli.cmd_coordinator and coord.port == 8111 and coord.store is None


def test_box_entrypoint_command_parses():
    out = _dry("entrypoint-box.sh", {"GPUS": "8", "PRESET": "large", "CHECKPOINT_STORE": "/ck", "RESUME": "1",
                                     "METRICS_PORT": "9400", "STEPS": "77"})
    line = out.strip().splitlines()[-1]
    toks = shlex.split(line)
    assert toks[1:3] == ["-m", "torch.distributed.run"]
    assert toks[toks.index("--nproc-per-node") + 1] == "8" and toks[toks.index("--master-addr") + 1] == "127.0.0.1"
    args = cli.build_parser().parse_args(_cli_args(line))
    assert args.fn is cli.cmd_train_box
    assert (args.preset, args.steps, args.checkpoint_store, args.resume, args.metrics_port) == \
        ("large", 77, "/ck", True, 9400)


def test_bootstrap_if_absent_and_env_store(tmp_path, monkeypatch, capsys):
    from distrain_b200 import protocol as P
    from distrain_b200.utils.storage import FsStore, S3Store
    store = str(tmp_path / "store")
    cli.main(["bootstrap", "--store", store, "--preset", "micro", "--seed", "0"])
    first = FsStore(store).get(P.checkpoint_path(0))
    cli.main(["bootstrap", "--store", store, "--preset", "micro", "--seed", "1", "--if-absent"])
    assert "bootstrap_skipped" in capsys.readouterr().out
    assert FsStore(store).get(P.checkpoint_path(0)) == first  # a second bootstrap (seed 1) would differ
    monkeypatch.setenv("R2_ENDPOINT", "http://objects.internal:9000")
    monkeypatch.setenv("R2_BUCKET", "runs")
    s = cli._store(None)
    assert isinstance(s, S3Store) and s.cfg.endpoint == "http://objects.internal:9000" and s.cfg.bucket == "runs"


@pytest.mark.skipif(shutil.which("make") is None, reason="make not installed")
def test_make_targets_expand():
    text = open(os.path.join(ROOT, "Makefile")).read()
    phony = re.search(r"^\.PHONY:((?:.*\\\n)*.*)$", text, re.M).group(1).replace("\\\n", " ").split()
    assert "build" in phony and "test" in phony
    for t in phony:
        r = subprocess.run(["make", "-n", "-C", ROOT, t], capture_output=True, text=True, timeout=60)
        assert r.returncode == 0, (t, r.stderr)
    ci = yaml.safe_load(open(os.path.join(ROOT, ".github/workflows/ci.yml")))
    runs = [st.get("run", "") for job in ci["jobs"].values() for st in job["steps"]]
    used = re.findall(r"(?:^|&& |\$PATH )make ([\w-]+)", "\n".join(runs), re.M)
    assert used and set(used) <= set(phony), used


def test_pyproject_entry_point_and_package_data():
    meta = tomllib.load(open(os.path.join(ROOT, "pyproject.toml"), "rb"))
    import distrain_b200
    assert meta["project"]["version"] == distrain_b200.__version__
    mod, fn = meta["project"]["scripts"]["distrain-b200"].split(":")
    assert getattr(importlib.import_module(mod), fn) is cli.main
    for pat in meta["tool"]["setuptools"]["package-data"]["distrain_b200"]:
        if not pat.startswith("lib/"):
            assert glob.glob(os.path.join(ROOT, "distrain_b200", pat)), pat

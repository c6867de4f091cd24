# Task runner: build, test, benchmarks, data, containers. GPU targets need a B200 (sm_100a).
PY ?= python
GPUS ?= 8
PORT ?= 29511
STEPS ?= 20
WARMUP ?= 3
IMAGE ?= distrain-b200:latest
TORCHRUN = timeout -k 60 1800 $(PY) -m torch.distributed.run --nnodes 1 --nproc-per-node $(GPUS) \
           --master-addr 127.0.0.1 --master-port $(PORT)

.PHONY: help build build-force test test-gpu selftest smoke bench bench-scale bench-merge bench-kernels \
        bench-loss data micro-cluster train-box docker compose-up compose-down lint clean

help:
	@grep -E '^[a-z-]+:.*## ' $(MAKEFILE_LIST) | sed 's/:.*## /\t/'

build: ## compile the sm_100a kernel library and the C++ runtime in-tree
	$(PY) -m distrain_b200._build

build-force: ## rebuild every object
	$(PY) -m distrain_b200._build --force

test: build ## CPU tests (includes multi-process gloo clusters)
	$(PY) -m pytest tests/ -x -q -m "not gpu"

test-gpu: build ## GPU tests (B200)
	$(PY) -m pytest tests/ -x -q -m gpu

selftest: ## native runtime self-test under ASan+UBSan and TSan
	$(PY) -m pytest tests/test_runtime_sanitizers.py -q

smoke: build ## one forward+backward of the flagship model on cuda:0
	$(PY) __graft_entry__.py smoke

bench: build ## headline benchmark on one GPU
	$(PY) bench.py --steps $(STEPS) --warmup $(WARMUP)

bench-scale: build ## headline benchmark on GPUS GPUs of this box
	$(TORCHRUN) bench.py --gpus $(GPUS) --steps $(STEPS) --warmup $(WARMUP)

bench-merge: build ## compress -> merge -> broadcast microbenchmark (GPUS nodes)
	$(TORCHRUN) -m distrain_b200.bench_merge

bench-kernels: build ## per-kernel times and roofline fractions (one GPU)
	$(PY) -m distrain_b200.bench_kernels --json

bench-loss: build ## loss gap to one GPU at matched tokens (2 nodes)
	$(MAKE) GPUS=2 _bench-loss
_bench-loss:
	$(TORCHRUN) -m distrain_b200.bench_loss --steps 300

data: ## random token shards + manifest in ./data (the data-prep script's test mode)
	$(PY) -m distrain_b200 prepare-data --output-dir data --num-shards 8 --tokens-per-shard 10000000

micro-cluster: ## coordinator + 2 CPU nodes over HTTP on the micro-test workload
	$(PY) -m distrain_b200 micro-cluster --nodes 2 --steps 60

train-box: build ## in-box training on GPUS GPUs (tiny preset, shards from ./data when present)
	$(TORCHRUN) -m distrain_b200 train-box --preset tiny --steps 1000 $(if $(wildcard data),--data-dir data,)

docker: ## container image for coordinator, HTTP nodes and the in-box job
	docker build -f deploy/Dockerfile -t $(IMAGE) .

compose-up: ## local stack: object store, coordinator, in-box job, Prometheus, Grafana
	docker compose -f deploy/compose.yml up -d

compose-down:
	docker compose -f deploy/compose.yml down

lint: ## byte-compile every module and rebuild the native libraries
	$(PY) -m compileall -q distrain_b200 tests bench.py
	$(PY) -m distrain_b200._build

clean: ## remove build objects and built libraries
	rm -rf _build distrain_b200/lib/*.so

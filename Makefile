# Entry points of the repository. Reference: Makefile:8-20 (lint lane, CPU test lane).
PY ?= python

.PHONY: build lint test-cpu test-gpu bench bench-reference quickstart

build:            ## compile every CUDA extension for sm_100a into the tree
	$(PY) -c "import __graft_entry__ as g; g.build()"

lint:             ## unbound names, source contracts (bounded spins, no traps, descriptor parity, ...)
	$(PY) -m pytest tests/test_static_names.py tests/test_kernel_source_contracts.py -q

test-cpu:         ## everything that needs no GPU (gloo ranks for the multi-process paths)
	CUDA_VISIBLE_DEVICES= $(PY) -m pytest tests -q -m "not gpu"

test-gpu:         ## on a B200; multi-GPU tests skip themselves when fewer GPUs are visible
	$(PY) -m pytest tests -q -m gpu

bench:            ## 1 GPU, Qwen3-30B-A3B shapes
	$(PY) bench.py

bench-reference:  ## the unmodified reference's colocated engine on the same configuration
	$(PY) bench.py --impl reference

quickstart:
	bash fastafd_b200/server/quickstart.sh

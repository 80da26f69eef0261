"""The served path on a GPU: HTTP -> tokenizer -> coordinator -> ZeroMQ -> one colocated GPU
worker process (CUDA graphs, fused kernels) and back. The greedy tokens that come back are
those of the same engine driven in-process by SpmdDriver."""
import pytest

from fastafd_b200.config import PRESETS, RuntimeConfig
from fastafd_b200.core import SamplingParams
from fastafd_b200.server.args import parse_args

pytestmark = pytest.mark.gpu
PROMPTS = [[5, 9, 200, 31, 77, 4], [1000, 3, 3, 8], list(range(40, 75))]


@pytest.mark.timeout(600)
def test_http_round_trip_on_one_gpu_matches_the_in_process_engine():
    from serving_util import greedy_tokens, running_server

    args = parse_args(["--mode", "serve", "--model-path", "tiny-qwen3-moe", "--device", "cuda", "--afd-num-mb", "2",
                       "--num-pages", "64", "--max-seq-len-override", "128", "--afd-max-running-requests", "8",
                       "--cuda-graph-max-bs", "8"])
    with running_server(args) as (base, sup):
        got = [greedy_tokens(base, p, 8) for p in PROMPTS]
        again = [greedy_tokens(base, p, 8) for p in PROMPTS]
        assert sup.get_failures() == []
    assert got == again

    from fastafd_b200.engine import AfdEngine, SpmdDriver
    from fastafd_b200.protocol import AfdTopology

    rt = args.runtime_config()
    eng = AfdEngine(PRESETS["tiny-qwen3-moe"], rt, AfdTopology(colocated=True), 0, "cuda:0", seed=args.seed, fast_init=True)   # the worker process draws its weights on the GPU too
    try:
        # one request at a time, like the HTTP calls above (same batch shapes, same kernels)
        expect = [SpmdDriver(eng).generate([p], SamplingParams(max_tokens=8, ignore_eos=True))[0] for p in PROMPTS]
    finally:
        eng.close()
    assert got == expect

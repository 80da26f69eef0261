"""Reference arm of the headline benchmark: the unmodified reference engine, stock code path.

The reference package (``minisgl``, installed under ``baseline/_ref``) is driven through its own
offline entry point ``minisgl.llm.LLM.generate`` (python/minisgl/llm/llm.py:28-98) on its colocated
engine (python/minisgl/engine/engine.py:212-433) with ``use_dummy_weight=True``
(python/minisgl/server/args.py:292-297): TRT-LLM-gen attention through FlashInfer, its Triton fused
MoE, its tvm-ffi JIT ops and its CUDA-graph runner.  Nothing of this repository's models, kernels or
engine is imported here.

What this file adds around the reference is measurement only:
  * a model directory with the ``config.json`` of the named architecture and a tiny word-level
    tokenizer (the reference loads both from disk; there is no checkpoint to download);
  * a wrapper around ``engine.forward_batch`` that records a CUDA event and a host time stamp at the
    start of every forward, so that the steady-state decode steps can be cut out of the run.

``value`` is the device time between the start of decode step W and the start of decode step W+K
(the reference's overlap scheduler keeps the GPU queue one step ahead of the host); ``e2e`` is the
wall clock between the same two points, which contains each step's pinned host-to-device copies and
the device-to-host read of the sampled tokens that the reference's scheduler performs.
The reference's AFD mode starts every worker as a Ray actor (python/minisgl/afd_coordinator.py:15);
Ray is not installed, so for N >= 2 the arm reports itself unavailable.
"""
from __future__ import annotations

import json
import os
import statistics
import sys
import tempfile
import time
import traceback

HERE = os.path.dirname(os.path.abspath(__file__))
REF_ROOT = os.path.join(HERE, "_ref")

HF_CONFIGS = {
    "qwen3-30b-a3b": {
        "architectures": ["Qwen3MoeForCausalLM"], "model_type": "qwen3_moe", "hidden_size": 2048,
        "num_hidden_layers": 48, "num_attention_heads": 32, "num_key_value_heads": 4, "head_dim": 128,
        "intermediate_size": 6144, "moe_intermediate_size": 768, "num_experts": 128, "num_experts_per_tok": 8,
        "norm_topk_prob": True, "vocab_size": 151936, "rms_norm_eps": 1e-6, "rope_theta": 1000000.0,
        "max_position_embeddings": 40960, "hidden_act": "silu", "tie_word_embeddings": False,
        "torch_dtype": "bfloat16", "decoder_sparse_step": 1, "mlp_only_layers": [], "attention_bias": False,
        "attention_dropout": 0.0, "router_aux_loss_coef": 0.001, "output_router_logits": False,
        "sliding_window": None, "use_sliding_window": False, "rope_scaling": None,
    },
}


def write_model_dir(path: str, model: str, layers: int = 0) -> None:
    """config.json of the architecture + a word-level tokenizer with an EOS token."""
    cfg = dict(HF_CONFIGS[model])
    if layers:
        cfg["num_hidden_layers"] = layers
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f)
    from tokenizers import Tokenizer
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import Whitespace

    vocab = {"<unk>": 0, "<eos>": 1}
    vocab.update({f"w{i}": i + 2 for i in range(254)})
    tok = Tokenizer(WordLevel(vocab, unk_token="<unk>"))
    tok.pre_tokenizer = Whitespace()
    tok.save(os.path.join(path, "tokenizer.json"))
    with open(os.path.join(path, "tokenizer_config.json"), "w") as f:
        json.dump({"tokenizer_class": "PreTrainedTokenizerFast", "eos_token": "<eos>", "unk_token": "<unk>",
                   "model_max_length": 1 << 20}, f)


def _unavailable(reason: str) -> dict:
    return {"impl": "reference", "unavailable": " ".join(reason.split())[:600]}


def run(args, clock_sampler_cls=None) -> dict:
    if args.gpus != 1:
        return _unavailable("the reference's AFD workers are Ray actors (minisgl/afd_coordinator.py imports ray) and Ray is "
                            "not installed; only its colocated engine (N=1) runs on this image")
    if args.model not in HF_CONFIGS:
        return _unavailable(f"no dummy-weight config for {args.model} in the reference arm")
    if not os.path.isdir(os.path.join(REF_ROOT, "minisgl")):
        return _unavailable("baseline/_ref is not installed")
    stage = "import"
    try:
        os.environ.setdefault("TVM_FFI_CACHE_DIR", os.path.join(REF_ROOT, ".tvm_ffi_cache"))
        os.environ.setdefault("HF_HUB_OFFLINE", "1")
        os.environ.setdefault("TRANSFORMERS_OFFLINE", "1")
        sys.path.insert(0, REF_ROOT)
        import torch
        from minisgl.core import SamplingParams
        from minisgl.llm import LLM

        b, ctx = args.batch_per_attn_gpu, args.context
        warm, steps = max(args.warmup, 3), args.steps
        n_decode = warm + steps + 4
        stage = "model directory"
        tmp = tempfile.mkdtemp(prefix="ref_model_")
        write_model_dir(tmp, args.model, getattr(args, "layers", 0))

        stage = "engine init (dummy weights, graph capture, JIT)"
        t0 = time.time()
        llm = LLM(tmp, dtype=torch.bfloat16, use_dummy_weight=True, max_running_req=b, cuda_graph_max_bs=b,
                  page_size=16, max_seq_len_override=ctx + n_decode + 64, max_extend_tokens=8192)
        build_s = time.time() - t0

        records = []          # (phase, size, event, host time)
        engine = llm.engine
        inner = engine.forward_batch

        def stamped(batch, sample_args):
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(engine.stream)
            records.append((batch.phase, batch.size, ev, time.perf_counter()))
            return inner(batch, sample_args)

        engine.forward_batch = stamped

        stage = "generate"
        gen = torch.Generator().manual_seed(1)
        prompts = torch.randint(2, 151936, (b, ctx), generator=gen).tolist()
        sp = SamplingParams(temperature=0.0, ignore_eos=True, max_tokens=n_decode)
        sampler = clock_sampler_cls(0) if clock_sampler_cls is not None else None
        if sampler is not None:
            sampler.start()
        outs = llm.generate(prompts, sp)
        torch.cuda.synchronize()
        clocks = sampler.stop() if sampler is not None else None

        stage = "timing"
        dec = [r for r in records if r[0] == "decode" and r[1] == b]
        if len(dec) < warm + steps + 1:
            return _unavailable(f"reference ran {len(dec)} full decode steps of batch {b}, need {warm + steps + 1}")
        first, last = dec[warm], dec[warm + steps]
        dev_ms = first[2].elapsed_time(last[2])
        e2e_ms = (last[3] - first[3]) * 1e3
        per_step = [dec[i][2].elapsed_time(dec[i + 1][2]) for i in range(warm, warm + steps)]
        tokens = b * steps
        n_out = [len(o["token_ids"]) for o in outs]
        # per decode step the reference's scheduler copies from pinned memory: positions (int32),
        # the token-pool row mapping (int64), the write mapping and write positions (2 x int64) and the
        # attention metadata (sequence lengths int32, cumulative lengths int32); it reads back the
        # sampled tokens (int32) after an event.
        h2d = b * 4 + b * 8 + 2 * b * 8 + b * 4 + (b + 1) * 4
        d2h = b * 4
        return {
            "impl": "reference",
            "metric": args.metric, "value": round(tokens / (dev_ms / 1e3), 2), "unit": "tok/s", "n_gpus": 1,
            "steps": steps, "warmup": warm, "ms_per_step": round(dev_ms / steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (reference dummy weights: torch.randn_like; random prompt ids)",
            "per_gpu_tok_s": round(tokens / (dev_ms / 1e3), 2),
            "tpot_p50_ms": round(statistics.median(per_step), 4),
            "config": {"model": args.model, "global_batch": b, "seq_len": ctx, "decode_tokens_timed": steps,
                       "parallelism": "colocated-1gpu", "page_size": 16, "attention_backend": "trtllm (auto)",
                       "moe_backend": "fused (auto)", "cuda_graph": True,
                       "l2": "per-step working set (expert weights + KV) is far larger than the 126 MB L2; no flush needed",
                       "prefill": f"{b} x {ctx} prompt tokens prefilled by the reference before the timed decode steps",
                       "output_tokens_per_request": [min(n_out), max(n_out)]},
            "clocks": clocks,
            "e2e": {"value": round(tokens / (e2e_ms / 1e3), 2), "unit": "tok/s", "ms_per_step": round(e2e_ms / steps, 4),
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "how": "wall clock of the same K decode steps inside LLM.generate (overlap scheduler): host scheduling, "
                           "pinned H2D of the step's indices and lengths, graph replay, D2H of the sampled tokens"},
            "gpu_launches": None,
            "build_s": round(build_s, 1),
        }
    except BaseException as e:  # the attempt's own text is the reason
        if isinstance(e, KeyboardInterrupt):
            raise
        tb = traceback.extract_tb(e.__traceback__)
        where = f"{os.path.basename(tb[-1].filename)}:{tb[-1].lineno}" if tb else "?"
        sys.stderr.write(traceback.format_exc())
        return _unavailable(f"reference colocated engine failed at stage '{stage}': {type(e).__name__}: {e} ({where})")

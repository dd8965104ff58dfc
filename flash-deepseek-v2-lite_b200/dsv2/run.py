"""Decode runner CLI: prefill once, capture one q_len=1 decode step in a CUDA graph, replay it.

    python -m dsv2.run [--model-path DIR] [--batch-size B | --batch-sizes "1 32 256"]
                       [--max-new-tokens N] [--kernel-family small|batch]
                       [--dump-token-ids] [--dump-step-trace]

Mirrors the reference runner (src/run.py:220-236 options, :591-688 harness, :690-757
output): greedy decode of one prompt replicated over the batch, the decode time taken
with perf_counter around graph replays 1..N-1 with a device sync at both ends, and one
JSON document with batch_size, path, ttft_ms, tps, decode_tokens (+ generated token ids /
per-step trace on request) and a hardware summary.

Model: ``--model-path`` loads a DeepSeek-V2-Lite checkpoint with transformers' native
DeepseekV2 classes (tokenizer + chat template for ``--prompt``).  Without it the runner
uses the seeded synthetic model of dsv2.synthetic and ``--prompt-len`` random token ids.
"""
from __future__ import annotations

import argparse
import json
import os
import platform
import time

import torch

from .engine import FAMILIES, DecodeEngine


def _parse_args(argv=None):
    ap = argparse.ArgumentParser(description="DeepSeek-V2-Lite decode on B200 kernels (libdsv2).")
    ap.add_argument("--model-path", type=str, default=None,
                    help="checkpoint directory; default: seeded synthetic DeepSeek-V2-Lite")
    ap.add_argument("--prompt", type=str, default="Write a short story about a lighthouse keeper.")
    ap.add_argument("--prompt-len", type=int, default=512, help="synthetic model: prompt length")
    ap.add_argument("--layers", type=int, default=27, help="synthetic model: decoder layers")
    ap.add_argument("--seed", type=int, default=1, help="synthetic model: weight seed")
    ap.add_argument("--max-new-tokens", type=int, default=128)
    ap.add_argument("--batch-size", type=int, default=1)
    ap.add_argument("--batch-sizes", type=str, default=None, help='Comma/space separated sweep, e.g. "1 2 4".')
    ap.add_argument("--kernel-family", choices=sorted(FAMILIES), default=None,
                    help="small (GEMV) or batch (tcgen05); default: small for B <= 4, else batch")
    ap.add_argument("--device", type=str, default="cuda:0")
    ap.add_argument("--prefill", choices=["kernels", "eager"], default="kernels",
                    help="prompt prefill through the decode kernels or the HF forward")
    ap.add_argument("--dump-token-ids", action="store_true")
    ap.add_argument("--dump-step-trace", action="store_true")
    return ap.parse_args(argv)


def _batch_sizes(args) -> list[int]:
    if args.batch_sizes:
        out = [int(x) for x in args.batch_sizes.replace(",", " ").split()]
    else:
        out = [args.batch_size]
    if not out or any(b <= 0 for b in out):
        raise ValueError("batch sizes must be positive")
    return out


def _load(args, dev):
    if args.model_path:
        from transformers import AutoModelForCausalLM, AutoTokenizer
        os.environ.setdefault("HF_HUB_OFFLINE", "1")
        os.environ.setdefault("TRANSFORMERS_OFFLINE", "1")
        tok = AutoTokenizer.from_pretrained(args.model_path)
        model = AutoModelForCausalLM.from_pretrained(args.model_path, dtype=torch.bfloat16,
                                                     attn_implementation="eager").to(dev).eval()
        ids = tok.apply_chat_template([{"role": "user", "content": args.prompt}], add_generation_prompt=True,
                                      return_tensors="pt")
        if not torch.is_tensor(ids):
            ids = ids["input_ids"]
        return model, ids.view(-1).to(dev)
    from .synthetic import build_model, dsv2_lite_config
    cfg = dsv2_lite_config(num_layers=args.layers)
    model = build_model(cfg, seed=args.seed, device=dev, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(args.seed + 1000)
    ids = torch.randint(0, cfg.vocab_size, (args.prompt_len,), generator=g)
    return model, ids.to(dev)


def hardware_info(dev: torch.device) -> dict:
    props = torch.cuda.get_device_properties(dev)
    try:
        import psutil
        cpu = {"physical_cores": psutil.cpu_count(logical=False), "logical_cores": psutil.cpu_count(logical=True),
               "memory_gb": round(psutil.virtual_memory().total / 1024 ** 3, 2)}
    except ImportError:  # pragma: no cover
        cpu = {"logical_cores": os.cpu_count()}
    return {
        "cpu": cpu,
        "gpu": {"visible_index": dev.index, "name": props.name, "capability": f"sm{props.major}{props.minor}",
                "sm_count": props.multi_processor_count, "memory_gb": round(props.total_memory / 1024 ** 3, 2)},
        "software": {"python": platform.python_version(), "torch": torch.__version__,
                     "torch_cuda": torch.version.cuda},
    }


def run_graph_decode(model, prompt: torch.Tensor, batch: int, max_new_tokens: int, family: str,
                     dump_token_ids: bool = False, dump_step_trace: bool = False,
                     prefill: str = "kernels") -> dict:
    """Prefill + graph decode of `prompt` replicated over `batch` rows; returns the
    reference runner's per-batch result fields."""
    dev = prompt.device
    prompt_len = int(prompt.numel())
    max_len = prompt_len + max_new_tokens + 8
    eng = DecodeEngine(model, batch, max_len, family)
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    first = eng.prefill([prompt] * batch, method=prefill)
    torch.cuda.synchronize(dev)
    prefill_s = time.perf_counter() - t0
    collect = dump_token_ids or dump_step_trace
    generated = [[int(t)] for t in first.cpu().tolist()] if collect else None
    trace: list[dict] = []

    def add_trace(step, toks, pos):
        if dump_step_trace:
            e = {"step": step, "cache_position": pos}
            if len(toks) == 1:
                e["token_id"] = toks[0]
            else:
                e["token_ids"] = toks
            trace.append(e)

    if generated is not None:
        add_trace(0, [g[0] for g in generated], prompt_len)
    eng.capture()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for step in range(1, max_new_tokens):
        eng.replay()
        if generated is not None:
            toks = [int(t) for t in eng.input_ids.cpu().tolist()]
            for row, t in enumerate(toks):
                generated[row].append(t)
            add_trace(step, toks, prompt_len + step)
    torch.cuda.synchronize(dev)
    decode_s = time.perf_counter() - t0
    eng.release()
    decode_tokens = batch * max(max_new_tokens - 1, 0)
    out = {"batch_size": batch, "path": f"dsv2_{family}_graph", "ttft_ms": prefill_s * 1000.0,
           "tps": decode_tokens / decode_s if decode_s > 0 else 0.0, "decode_tokens": decode_tokens}
    if dump_token_ids:
        out["generated_token_ids"] = generated[0] if batch == 1 else generated
    if dump_step_trace:
        out["step_trace"] = trace
    return out


def main(argv=None) -> None:
    args = _parse_args(argv)
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is required for this benchmark")
    dev = torch.device(args.device)
    torch.cuda.set_device(dev)
    model, prompt = _load(args, dev)
    results = []
    for b in _batch_sizes(args):
        family = args.kernel_family or ("small" if b <= 4 else "batch")
        results.append(run_graph_decode(model, prompt, b, args.max_new_tokens, family,
                                        args.dump_token_ids, args.dump_step_trace, prefill=args.prefill))
    hw = hardware_info(dev)
    doc = dict(results[0], hardware=hw) if len(results) == 1 else {"results": results, "hardware": hw}
    print(json.dumps(doc, ensure_ascii=False, indent=2))


if __name__ == "__main__":
    main()

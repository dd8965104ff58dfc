"""Decode throughput benchmark for the B200 DeepSeek-V2-Lite engine.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2|3|4|5] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N   (expert parallel)

Workload (synthetic seeded inputs stand in for real prompts):
  config 2: 27-layer DeepSeek-V2-Lite, bf16 N(0, 0.02) weights seed 1, B=1, 512-token prompt, small family
  config 3: same weights, B=32, 512-token prompts (seed 2), batch family
  config 4: same weights, B=256, prompt lengths U[128, 1024] (seed 3), ragged latent cache, batch family
            (default: the north-star roofline target and the largest single-GPU config)
  config 5: same weights, B=64, 8192-token prompts (seed 4), Zipf(1.1)-skewed router
One step = one CUDA-graph replay of the q_len=1 decode step for every row (all 27
layers, lm_head and greedy argmax).  `value` = decoded tokens / s over all ranks, timed
with CUDA events over K replays (max over ranks); the per-step working set (~31 GB of
weights) is far larger than L2, so no flush is needed between steps.  `e2e` repeats the
decode through the public engine API with the token ids crossing host<->device every
step (pinned buffers, copies inside the timed region).  The default single-GPU run also
summarises configs 3 and 2 (B=32, B=1) under "other_configs".  `cpu_baseline` and the
`--impl reference` arm run the same routine: the reference's CPU path (HF eager bf16) on
the host cores for the whole workload batch, per-layer times measured on a 2-layer slice.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import threading
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "flash-deepseek-v2-lite_b200"))
sys.path.insert(0, str(REPO))

METRIC = "decode tok/s at bsz 1/32/256, ctx 512; ms/step vs HBM roofline; 1/2/4/8 GPU"

CONFIGS = {
    2: dict(batch=1, prompt=("fixed", 512), seed=1, family="small", skew=False),
    3: dict(batch=32, prompt=("fixed", 512), seed=2, family="batch", skew=False),
    4: dict(batch=256, prompt=("uniform", 128, 1024), seed=3, family="batch", skew=False),
    5: dict(batch=64, prompt=("fixed", 8192), seed=4, family="batch", skew=True),
}
WEIGHT_SEED = 1

# algorithmic bytes per step: bf16 weights read once (attention, dense MLP, shared experts,
# gate, lm_head, distinct routed experts) + the latent KV rows attended
ATTN_BYTES = 2 * 13_767_168
DENSE_BYTES = 2 * 67_239_936
SHARED_BYTES = 2 * 17_301_504
GATE_BYTES = 2 * 131_072
LMHEAD_BYTES = 2 * 209_715_200
EXPERT_BYTES = 2 * 8_650_752
KV_ROW_BYTES = 576 * 2
# DRAM traffic / algorithmic bytes of the fused MoE launch, from one ncu capture of the
# current kernel at B=256 (all 64 experts hit; profiles/moe_tc_b256.md):
# (1159.24 + 21.20) MB / 1141.90 MB
MOE_TRAFFIC_RATIO = 1.0337
MOE_TRAFFIC_SOURCE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one fused MoE launch "
                      "(dsv2.microbench moe, B=256, all 64 experts hit; profiles/moe_tc_b256.md), "
                      "scaled to this launch by its algorithmic bytes")


def prompt_lengths(cfg: dict, batch: int) -> list[int]:
    kind = cfg["prompt"][0]
    if kind == "fixed":
        return [cfg["prompt"][1]] * batch
    g = torch.Generator().manual_seed(cfg["seed"])
    lo, hi = cfg["prompt"][1], cfg["prompt"][2]
    return torch.randint(lo, hi + 1, (batch,), generator=g).tolist()


def make_prompts(cfg: dict, batch: int, vocab: int) -> list[torch.Tensor]:
    lens = prompt_lengths(cfg, batch)
    g = torch.Generator().manual_seed(cfg["seed"] + 1000)
    return [torch.randint(0, vocab, (n,), generator=g) for n in lens]


class ClockSampler:
    """Samples SM clock and throttle reasons with NVML every 200 ms (read-only)."""

    def __init__(self, index: int):
        self.samples: list[tuple[float, float, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM))
        except Exception:
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                reasons = int(nv.nvmlDeviceGetCurrentClocksEventReasons(self._h))
                util = float(nv.nvmlDeviceGetUtilizationRates(self._h).gpu)
                self.samples.append((sm, util, reasons))
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        if self._nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t is not None:
            self._t.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        nv = self._nv
        names = {
            "sw_power_cap": getattr(nv, "nvmlClocksEventReasonSwPowerCap", 0x4),
            "hw_slowdown": getattr(nv, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "sw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "hw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "hw_power_brake_slowdown": getattr(nv, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
        }
        load = [s for s in self.samples if s[1] > 0] or self.samples
        mhz = sorted(s[0] for s in load)
        seen = 0
        for s in load:
            seen |= s[2]
        return {"sm_mhz": mhz[len(mhz) // 2], "sm_max_mhz": self.max_mhz,
                "reasons": [k for k, bit in names.items() if seen & bit], "samples": len(load)}


def measured_peak() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def init_dist(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
        return rank, world, local, dist.group.WORLD
    if torch.cuda.is_available():
        torch.cuda.set_device(0)
    return 0, 1, 0, None


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def count_launches(fn) -> int:
    """Number of libdsv2 kernels one call of fn enqueues (the library's own launch counter)."""
    from dsv2 import _lib
    n0 = _lib.kernel_launches()
    fn()
    return _lib.kernel_launches() - n0


def step_bytes(eng, lens_now: list[int], distinct: list[int]) -> float:
    """Algorithmic HBM bytes of one decode step on this rank (weights read once + latent KV)."""
    n_moe = len(distinct)
    n_dense = eng.L - n_moe
    b = eng.L * ATTN_BYTES + n_dense * DENSE_BYTES + n_moe * (SHARED_BYTES + GATE_BYTES) + LMHEAD_BYTES
    b += sum(distinct) * EXPERT_BYTES
    b += sum(lens_now) * eng.L * KV_ROW_BYTES
    return float(b)


def distinct_experts(eng) -> list[int]:
    go = eng.group_offsets_hist.cpu()
    counts = go[:, 1:eng.n_groups - 1] - go[:, :eng.n_groups - 2]
    return [int((c > 0).sum()) for c in counts]


def build_engine_for(model, cfg_id: int, B_all: int, family: str, rank: int, world: int, group, args,
                     steps_total: int, bias):
    from dsv2.engine import DecodeEngine
    cfg = CONFIGS[cfg_id]
    B = B_all // world
    prompts_all = make_prompts(cfg, B_all, model.config.vocab_size)
    prompts = prompts_all[rank * B:(rank + 1) * B]
    max_len = max(len(p) for p in prompts_all) + steps_total + 8
    eng = DecodeEngine(model, B, max_len, family, rank=rank, world=world, group=group, gate_bias=bias)
    return eng, prompts


def measure(model, cfg_id: int, args, rank: int, world: int, group, local: int, bias, steps: int, warmup: int,
            e2e_steps: int, family: str | None = None, batch: int | None = None, clocks_out: dict | None = None):
    """Prefill, capture and time one configuration on this rank's GPU (max over ranks).
    Returns the measured figures (whole-job tok/s, ms/step, step roofline, e2e, launches)."""
    cfg = CONFIGS[cfg_id]
    B_all = batch or cfg["batch"]
    if B_all % world:
        raise SystemExit(f"batch {B_all} not divisible by {world} ranks")
    family = family or cfg["family"]
    t0 = time.time()
    eng, prompts = build_engine_for(model, cfg_id, B_all, family, rank, world, group, args,
                                    warmup + steps + e2e_steps + 8, bias)
    t_build = time.time() - t0
    t0 = time.time()
    eng.prefill(prompts, max_tokens_per_chunk=args.prefill_chunk, method=args.prefill)
    torch.cuda.synchronize()
    t_prefill = time.time() - t0
    launches_per_step = count_launches(lambda: (eng.step(), eng.restore()))
    eng.capture()
    barrier(world)
    for _ in range(warmup):
        eng.replay()
    lens_before = [int(x) for x in eng.positions.cpu()]
    if getattr(eng, "peer_wait_stats", None) is not None:
        eng.peer_wait_stats.zero_()
    barrier(world)
    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        torch.cuda.nvtx.range_push("dsv2_timed")  # lets ncu --nvtx-include select the timed steps
        start.record(stream)
        for _ in range(steps):
            eng.replay()
        end.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    barrier(world)
    ms_rank = start.elapsed_time(end)
    per_rank = None
    if world > 1:
        # per-rank step time and the cross-GPU waits (mean CTA wait of a launch x MoE layers)
        import torch.distributed as dist
        waits = None
        if getattr(eng, "peer_wait_stats", None) is not None:
            st = [int(v) for v in eng.peer_wait_stats.cpu()]
            n_moe = int(eng.peers.n_moe_layers)
            waits = {"dispatch_wait_us_per_step": round(st[0] / max(st[1], 1) * n_moe / 1e3, 2),
                     "combine_wait_us_per_step": round(st[2] / max(st[3], 1) * n_moe / 1e3, 2)}
        per_rank = [None] * world
        dist.all_gather_object(per_rank, {"rank": rank, "ms_per_step": round(ms_rank / steps, 4), **(waits or {})})
    ms = max_over_ranks(ms_rank, world)
    ms_step = ms / steps
    value = B_all * steps / (ms / 1000.0)
    distinct = distinct_experts(eng)
    lens_mid = [l + steps // 2 for l in lens_before]
    bytes_rank = max_over_ranks(step_bytes(eng, lens_mid, distinct), world)
    peak, peak_kind = measured_peak()
    step_gbs = bytes_rank / (ms_step / 1000.0) / 1e9
    if clocks_out is not None:
        clocks_out.update(clocks.summary())

    # end to end through the public API: token ids cross host<->device every step
    B = B_all // world
    pin_in = torch.zeros(B, dtype=torch.int64, pin_memory=True)
    pin_out = torch.zeros(B, dtype=torch.int64, pin_memory=True)
    pin_in.copy_(eng.input_ids.cpu())
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_e2e = time.perf_counter()
    e0.record(stream)
    for _ in range(e2e_steps):
        eng.input_ids.copy_(pin_in, non_blocking=True)
        eng.replay()
        pin_out.copy_(eng.next_ids, non_blocking=True)
        stream.synchronize()
        pin_in.copy_(pin_out)
    e1.record(stream)
    torch.cuda.synchronize()
    t_e2e = time.perf_counter() - t_e2e
    e2e_s = max_over_ranks(max(t_e2e, e0.elapsed_time(e1) / 1000.0), world)
    res = {
        "eng": eng, "B_all": B_all, "family": family, "value": value, "ms_step": ms_step,
        "bytes_rank": bytes_rank, "step_gbs": step_gbs, "peak": peak, "peak_kind": peak_kind,
        "distinct": distinct, "launches_per_step": launches_per_step, "lens_before": lens_before,
        "e2e_value": B_all * e2e_steps / e2e_s, "e2e_bytes": 8 * B_all,
        "t_build": t_build, "t_prefill": t_prefill, "prefill_tokens": sum(len(p) for p in prompts),
        "per_rank": per_rank,
    }
    return res


def summary_of(res: dict, steps: int) -> dict:
    return {"value": round(res["value"], 2), "unit": "tok/s", "ms_per_step": round(res["ms_step"], 4),
            "steps": steps, "global_batch": res["B_all"], "kernel_family": res["family"],
            "step_roofline_frac": round(res["step_gbs"] / res["peak"], 4),
            "algorithmic_bytes_per_step": res["bytes_rank"],
            "distinct_experts_mean": round(sum(res["distinct"]) / max(len(res["distinct"]), 1), 2),
            "launches_per_step": res["launches_per_step"],
            "e2e_value": round(res["e2e_value"], 2)}


def run_ours(args, cfg_id: int):
    from dsv2.synthetic import add_router_bias, build_model, dsv2_lite_config, router_bias_zipf

    rank, world, local, group = init_dist(args)
    dev = torch.device("cuda", local)
    cfg = CONFIGS[cfg_id]
    t0 = time.time()
    mcfg = dsv2_lite_config(num_layers=args.layers)
    model = build_model(mcfg, seed=WEIGHT_SEED, device=dev, dtype=torch.bfloat16)
    bias = router_bias_zipf(mcfg.n_routed_experts, 1.1, seed=4).to(dev) if cfg["skew"] else None
    if bias is not None:
        add_router_bias(model, bias)
    t_model = time.time() - t0
    clocks = {}
    res = measure(model, cfg_id, args, rank, world, group, local, bias, args.steps, args.warmup, args.e2e_steps,
                  family=args.family, batch=args.batch, clocks_out=clocks)
    eng = res["eng"]
    B_all, family, ms_step = res["B_all"], res["family"], res["ms_step"]
    peak, peak_kind = res["peak"], res["peak_kind"]

    # dominant kernel: grouped MoE GEMMs (gate_up+SwiGLU and down) of all MoE layers,
    # replayed alone from a graph with the last routing in place
    moe_ms, moe_bytes, moe_launches = eng.time_moe_gemms(iters=max(3, min(args.steps, 20)))
    moe_ms = max_over_ranks(moe_ms, world)
    dk_gbs = moe_bytes / (moe_ms / 1000.0) / 1e9 if moe_ms > 0 else None
    lens_before = res["lens_before"]
    split_len = eng.split_len
    eng.release()
    barrier(world)
    eng.close()
    del eng, res["eng"]
    torch.cuda.empty_cache()

    # the other single-GPU configurations of the metric (B=32 batch family, B=1 small
    # family), summarised beside the headline
    extra = {}
    if world == 1 and cfg_id == 4 and not args.no_extra_configs and args.batch is None and args.family is None:
        for cid in (3, 2):
            n = min(args.steps, 20)
            r = measure(model, cid, args, rank, world, group, local, None, n, 3, 5)
            r["eng"].release()
            r["eng"].close()
            del r["eng"]
            torch.cuda.empty_cache()
            extra[f"config{cid}"] = summary_of(r, n)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_decode_baseline(cfg_id, B_all, args.layers, steps=2)
        cpu = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
    out = None
    if rank == 0:
        out = {
            "metric": METRIC,
            "value": round(res["value"], 2),
            "unit": "tok/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic: seeded random-init N(0,0.02) bf16 weights, seeded uniform random prompt ids",
            "config": {
                "workload": f"config {cfg_id}: DeepSeek-V2-Lite {args.layers} layers, batch {B_all}, "
                            f"prompts {cfg['prompt']}, {family} kernel family, CUDA-graph q_len=1 decode",
                "global_batch": B_all,
                "seq_len": int(sum(lens_before) / len(lens_before)),
                "parallelism": f"ep{world}+dp{world}" if world > 1 else "single",
                "kernel_family": family,
                "l2": "inputs larger than L2 (31 GB of weights streamed per step)",
                "split_len": split_len,
            },
            "roofline": {
                "bound": "hbm",
                "kernel": ("moe_tc_kernel: fused grouped MoE gate_up+SwiGLU+down (all MoE layers)"
                           if family == "batch" else
                           "gemv_mma_kernel: grouped MoE gate_up+SwiGLU and down (all MoE layers)"),
                "achieved": round(dk_gbs, 1) if dk_gbs else None,
                "peak": peak,
                "unit": "GB/s",
                "frac": round(dk_gbs / peak, 4) if dk_gbs else None,
                "peak_kind": peak_kind,
                "traffic": round(moe_bytes / max(moe_launches, 1) * MOE_TRAFFIC_RATIO),
                "traffic_source": MOE_TRAFFIC_SOURCE,
                "algorithmic_bytes_per_launch": round(moe_bytes / max(moe_launches, 1)),
                "launch_ms": round(moe_ms / max(moe_launches, 1), 5),
            },
            "step_roofline": {
                "algorithmic_bytes_per_step": res["bytes_rank"],
                "achieved": round(res["step_gbs"], 1),
                "peak": peak,
                "unit": "GB/s",
                "frac": round(res["step_gbs"] / peak, 4),
                "distinct_experts_mean": round(sum(res["distinct"]) / max(len(res["distinct"]), 1), 2),
            },
            "e2e": {"value": round(res["e2e_value"], 2), "unit": "tok/s", "h2d_bytes_per_step": res["e2e_bytes"],
                    "d2h_bytes_per_step": res["e2e_bytes"], "steps": args.e2e_steps},
            "gpu_launches": res["launches_per_step"] * args.steps,
            "launches_per_step": res["launches_per_step"],
            "clocks": clocks,
            "cpu_baseline": cpu,
            "other_configs": extra or None,
            "per_rank": res["per_rank"],
            "setup_s": {"model": round(t_model, 1), "engine": round(res["t_build"], 1),
                        "prefill": round(res["t_prefill"], 1), "prefill_method": args.prefill,
                        "prefill_tokens": res["prefill_tokens"]},
        }
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return out


def cpu_decode_baseline(cfg_id: int, B_all: int, layers: int, steps: int = 2) -> dict:
    """The reference's CPU path, HF eager bf16 (transformers 5.5) on the host cores, timed on
    a bounded sample of the workload: every row of the batch decodes together (one batch,
    prompts left-padded, the KV cache of each row filled to its prompt length with values
    that do not affect the cost), through a 2-layer slice of the model (the dense layer 0
    and one MoE layer, with the embedding, final norm and lm_head).  The layers are timed
    separately with forward hooks; the full-depth step is the measured
    rest + dense layer + (layers - 1) x MoE layer (the 26 MoE layers have identical shapes).
    Shared by bench.py's cpu_baseline and its --impl reference arm."""
    from transformers import StaticCache

    from oracle.hf_model import build_model, dsv2_lite_config
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = CONFIGS[cfg_id]
    mcfg = dsv2_lite_config(num_layers=2)
    t0 = time.perf_counter()
    model = build_model(mcfg, seed=WEIGHT_SEED, device="cpu", dtype=torch.float32).to(torch.bfloat16)
    t_build = time.perf_counter() - t0
    lens = prompt_lengths(cfg, B_all)
    R, T0 = len(lens), max(lens)
    g = torch.Generator().manual_seed(7)
    cache = StaticCache(config=mcfg, max_cache_len=T0 + steps + 1)
    heads = mcfg.num_attention_heads
    for li in range(2):
        k = (0.1 * torch.randn(R, heads, T0, mcfg.qk_nope_head_dim + mcfg.qk_rope_head_dim, generator=g)).to(torch.bfloat16)
        v = (0.1 * torch.randn(R, heads, T0, mcfg.v_head_dim, generator=g)).to(torch.bfloat16)
        cache.update(k, v, li, {"cache_position": torch.arange(T0)})
        del k, v
    mask = torch.zeros(R, T0 + steps + 1, dtype=torch.long)
    for r, n in enumerate(lens):
        mask[r, T0 - n:] = 1
    mask[:, T0:] = 1
    times: dict[str, list[float]] = {"layer0": [], "layer1": [], "total": []}
    marks = {}

    def pre(name):
        def f(*_a, **_k):
            marks[name] = time.perf_counter()
        return f

    def post(name):
        def f(*_a, **_k):
            times[name].append(time.perf_counter() - marks[name])
        return f
    hooks = []
    for i, layer in enumerate(model.model.layers):
        hooks.append(layer.register_forward_pre_hook(pre(f"layer{i}")))
        hooks.append(layer.register_forward_hook(post(f"layer{i}")))
    tok = torch.randint(0, mcfg.vocab_size, (R, 1), generator=g)
    with torch.no_grad():
        for s in range(steps + 1):          # the first step is an untimed warm-up
            pos = (torch.tensor(lens) + s).view(R, 1)
            t = time.perf_counter()
            out = model(input_ids=tok, attention_mask=mask[:, :T0 + s + 1], position_ids=pos,
                        past_key_values=cache, cache_position=torch.tensor([T0 + s]), use_cache=True)
            tok = out.logits[:, -1:].argmax(-1)
            times["total"].append(time.perf_counter() - t)
    for h in hooks:
        h.remove()

    def med(xs):
        xs = sorted(xs[1:])
        return xs[len(xs) // 2]
    t_l0, t_l1, t_tot = med(times["layer0"]), med(times["layer1"]), med(times["total"])
    t_rest = max(t_tot - t_l0 - t_l1, 0.0)
    step_full = t_rest + t_l0 + (layers - 1) * t_l1
    value = B_all / step_full
    sample = (f"HF eager bf16 (transformers 5.5) on {threads} host threads: all {R} rows of config {cfg_id} decoding "
              f"as one batch (left-padded to {T0}, static KV cache at each row's prompt length), {steps} timed "
              f"steps of a 2-layer slice; per step: dense layer {t_l0 * 1e3:.1f} ms, MoE layer {t_l1 * 1e3:.1f} ms, "
              f"embedding + final norm + lm_head {t_rest * 1e3:.1f} ms; full depth = rest + dense + "
              f"{layers - 1} MoE layers = {step_full * 1e3:.1f} ms")
    return {"value": round(value, 4), "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample,
            "ms_per_step": step_full * 1000.0, "build_s": round(t_build, 1)}


def run_reference(args, cfg_id: int):
    """Reference arm: the reference's CPU path (HF eager torch) on the host cores, through
    the same routine as the GPU arm's cpu_baseline; every step of the arm decodes the whole
    workload batch (steps of the routine = the arm's steps)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    cfg = CONFIGS[cfg_id]
    B_all = args.batch or cfg["batch"]
    r = cpu_decode_baseline(cfg_id, B_all, args.layers, steps=max(1, min(args.steps, 4)))
    value = r["value"]
    return {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(r["ms_per_step"], 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"config {cfg_id}: DeepSeek-V2-Lite {args.layers} layers, batch {B_all}, "
                               f"prompts {cfg['prompt']}", "global_batch": B_all, "parallelism": "cpu"},
        "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=4, choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=None, help="override the config's global batch")
    ap.add_argument("--family", default=None, choices=["small", "batch"])
    ap.add_argument("--layers", type=int, default=27)
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--prefill-chunk", type=int, default=4096)
    ap.add_argument("--prefill", default="kernels", choices=["kernels", "eager"],
                    help="prompt prefill: the decode kernels over token batches, or the HF forward")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra-configs", action="store_true",
                    help="skip the config 3 (B=32) and config 2 (B=1) summaries of the default run")
    args = ap.parse_args()
    if args.impl == "reference":
        out = run_reference(args, args.config)
    else:
        out = run_ours(args, args.config)
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()

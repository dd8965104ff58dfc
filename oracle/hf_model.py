"""Oracle model: the Hugging Face eager DeepSeek-V2 (transformers 5.5.0) with seeded weights.

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and the
CPU-baseline / reference arms of bench.py as the checker, never by the decode engine.

The reference (Flash-DeepSeeek-V2-Lite) loads DeepSeek-V2-Lite-Chat with the
checkpoint's remote modeling code (src/run.py:719-725), which is not available
here; its in-container stand-in is transformers' native
models/deepseek_v2/modeling_deepseek_v2.py (a third-party dependency, version
5.5.0), run eagerly.  The config and the seeded weight fill are the package's
synthetic-model builder (dsv2.synthetic), re-exported here, so the oracle and the
engine under test are built from identical weights by construction; what the oracle
adds is running the HF modules themselves (attention, experts, router) in eager mode.
"""
from __future__ import annotations

from dsv2.synthetic import YARN, add_router_bias, build_model, dsv2_lite_config, router_bias_zipf

__all__ = ["YARN", "dsv2_lite_config", "build_model", "router_bias_zipf", "add_router_bias"]

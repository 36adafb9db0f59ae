"""One typed engine configuration: CLI flags, a JSON/YAML file, or both.

Replaces the reference's mix of vLLM flags, ``--additional_config`` JSON and
30+ environment variables (``kernel-optimizations-recipe/
dsv41-flash-v6e16-serving.yaml:160-210,360-373``; runner argparse
``tpu-v7x/deepseek_v41/runner.py:813-823``).  Precedence: defaults < file <
flags.  ``to_dict()`` is echoed into every result JSON and ``/health`` so a
number always carries the configuration that produced it.  Environment
variables are read only for debug switches (``DSV4_TRACE_*``).
"""

from __future__ import annotations

import argparse
import dataclasses
import json
from dataclasses import dataclass, field


@dataclass
class EngineConfig:
    model: str = "v4-flash"                 # named config or a config.json path
    checkpoint: str | None = None           # safetensors directory (None: random init)
    preshard_dir: str | None = None         # per-rank pre-sharded blobs
    tokenizer: str | None = None            # HF tokenizer directory (None: byte tokenizer)
    served_model_name: str = "deepseek-v4-flash"
    device: str = "cuda"                    # "cuda" or "cpu" (the oracle test backend)
    seed: int = 0
    max_seqs: int = 512                     # --max-num-seqs
    max_batched_tokens: int = 1024          # --max-num-batched-tokens
    chunk_size: int | None = None           # prefill chunk (default: the token budget)
    max_model_len: int = 16384
    kv_block: int = 0                       # paged compressed caches: entries per block (0: per-slot caches)
    kv_pool_tokens: int = 0                 # paged pool size in tokens of context (0: max_seqs * max_model_len)
    gpu_memory_utilization: float | None = None  # paged caches without kv_pool_tokens: size the pool to
                                            # fill this fraction of the GPU's memory (vLLM's flag)
    kv_preempt: bool = False                # paged caches: admit on the prompt's blocks, preempt (recompute)
                                            # the newest request when the pool runs short
    use_cuda_graphs: bool = True
    expert_storage_layers: int | None = None
    ep_transport: str = "nccl"              # "nccl" (baseline), "p2p" (NVLink peer stores) or "fused"
                                            # (dispatch into the owners' expert rows, rows returned by W2)
    parallel: str = "ep"                    # multi-GPU layout: "ep" (data-parallel attention + expert
                                            # parallelism, throughput) or "tp" (tensor-parallel, latency)
    moe_split: str = "ep"                   # parallel="tp": experts owned whole ("ep") or split by
                                            # intermediate index over every GPU ("tp")
    dspark: bool = False                    # speculative decoding (DSpark 1+4, greedy; one GPU)
    dspark_force_accept: int | None = None
    engram_host_tables: bool = True
    engram_shm: str | None = None           # random-init Engram tables in shared files (e.g. /dev/shm/dsv4_engram)
    control_plane: str = "shm"              # multi-rank control messages: "shm" (one node, shared memory)
                                            # or "gloo" (the CPU process group)
    host: str = "127.0.0.1"
    api_key: str | None = None              # bearer key the API requires (or DSV4_API_KEY); None: open
    port: int = 8000
    step_deadline_s: float = 600.0
    drain_timeout_s: float = 30.0           # on SIGTERM: refuse new requests, let live ones finish this long
    overrides: dict = field(default_factory=dict)   # ModelConfig field overrides

    def to_dict(self) -> dict:
        """The fields as a dict (echoed into results and ``/health``), the API key redacted."""
        d = dataclasses.asdict(self)
        if d.get("api_key"):
            d["api_key"] = "(set)"
        return d

    def model_config(self):
        from ..config import ModelConfig, get_config

        if self.model.endswith(".json"):
            return ModelConfig.from_json(self.model, **self.overrides)
        return get_config(self.model, **self.overrides)

    @classmethod
    def from_file(cls, path: str) -> dict:
        with open(path) as f:
            if path.endswith((".yaml", ".yml")):
                import yaml
                return yaml.safe_load(f) or {}
            return json.load(f)

    @classmethod
    def parser(cls) -> argparse.ArgumentParser:
        p = argparse.ArgumentParser(description="DeepSeek-V4 family engine on B200")
        p.add_argument("--config-file", default=None, help="JSON or YAML file of EngineConfig fields")
        for f in dataclasses.fields(cls):
            if f.name == "overrides":
                p.add_argument("--override", action="append", default=None, metavar="KEY=JSON",
                               help="ModelConfig field override, e.g. --override n_layers=4")
                continue
            flag = "--" + f.name.replace("_", "-")
            if f.type in ("bool", bool):
                p.add_argument(flag, default=None, action=argparse.BooleanOptionalAction)
            else:
                typ = {"int": int, "float": float}.get(str(f.type).split(" ")[0], str)
                if "int |" in str(f.type):
                    typ = int
                p.add_argument(flag, default=None, type=typ)
        return p

    @classmethod
    def from_args(cls, argv: list[str] | None = None) -> "EngineConfig":
        a = cls.parser().parse_args(argv)
        vals: dict = {}
        if a.config_file:
            vals.update(cls.from_file(a.config_file))
        for f in dataclasses.fields(cls):
            if f.name == "overrides":
                continue
            v = getattr(a, f.name)
            if v is not None:
                vals[f.name] = v
        ov = dict(vals.pop("overrides", {}) or {})
        for kv in a.override or []:
            k, v = kv.split("=", 1)
            ov[k] = json.loads(v)
        unknown = set(vals) - {f.name for f in dataclasses.fields(cls)}
        if unknown:
            raise ValueError(f"unknown EngineConfig fields: {sorted(unknown)}")
        return cls(**vals, overrides=ov)

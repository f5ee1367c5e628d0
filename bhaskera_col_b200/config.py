"""KV-cache configuration keys of bhaskera (the subset this package serves).

Mirrors aditya25058/Bhaskera_col src/bhaskera/config.py:49-55 (TurboQuantConfig),
:98-111 (InferenceConfig) and the YAML parsing of ``inference.kv_cache`` /
``inference.turboquant.*`` at :425-440, so a bhaskera YAML file selects the
same cache here.  ``qjl`` is an added key (default off) that the reference
ignores.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, field
from typing import Any, Dict

import yaml


@dataclass
class TurboQuantConfig:
    enabled: bool = False
    key_bits: int = 4
    value_bits: int = 2
    residual_window: int = 128
    protected_layers: int = 2
    qjl: bool = False


@dataclass
class InferenceConfig:
    max_new_tokens: int = 512
    batch_size: int = 1
    kv_cache: str = "static"
    device: str = "auto"
    turboquant: TurboQuantConfig = field(default_factory=TurboQuantConfig)


@dataclass
class Config:
    inference: InferenceConfig = field(default_factory=InferenceConfig)

    def as_dict(self) -> Dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "Config":
        return _dict_to_config(d or {})


def _dict_to_config(raw: Dict[str, Any]) -> Config:
    inf = (raw or {}).get("inference") or {}
    tq = inf.get("turboquant") or {}
    return Config(inference=InferenceConfig(
        max_new_tokens=int(inf.get("max_new_tokens", 512)),
        batch_size=int(inf.get("batch_size", 1)),
        kv_cache=str(inf.get("kv_cache", "static")),
        device=str(inf.get("device", "auto")),
        turboquant=TurboQuantConfig(
            enabled=bool(tq.get("enabled", False)),
            key_bits=int(tq.get("key_bits", 4)),
            value_bits=int(tq.get("value_bits", 2)),
            residual_window=int(tq.get("residual_window", 128)),
            protected_layers=int(tq.get("protected_layers", 2)),
            qjl=bool(tq.get("qjl", False)),
        ),
    ))


def load_config(path: str) -> Config:
    with open(path) as f:
        raw = yaml.safe_load(f) or {}
    return _dict_to_config(raw)

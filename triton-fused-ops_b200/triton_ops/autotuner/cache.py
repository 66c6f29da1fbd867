"""JSON-backed cache of chosen configurations (API of the reference's ConfigCache)."""

import hashlib
import json
from pathlib import Path
from typing import Any, Dict, Optional, Tuple


class ConfigCache:
    """Maps (kernel_type, problem_size, device) to a configuration dict.

    With `cache_dir`, entries are also written to ``<cache_dir>/<key>.json``.
    """

    def __init__(self, cache_dir: Optional[str] = None):
        self.cache_dir = Path(cache_dir) if cache_dir else None
        self._memory_cache: Dict[str, Dict[str, Any]] = {}
        if self.cache_dir:
            self.cache_dir.mkdir(parents=True, exist_ok=True)

    @staticmethod
    def _make_key(kernel_type: str, problem_size: Tuple[int, ...], device: str) -> str:
        return hashlib.sha256(f"{kernel_type}|{tuple(problem_size)}|{device}".encode()).hexdigest()[:32]

    def get(self, kernel_type: str, problem_size: Tuple[int, ...], device: str) -> Optional[Dict[str, Any]]:
        key = self._make_key(kernel_type, problem_size, device)
        if key in self._memory_cache:
            return dict(self._memory_cache[key])
        if self.cache_dir:
            f = self.cache_dir / f"{key}.json"
            if f.exists():
                try:
                    cfg = json.loads(f.read_text())["config"]
                except (OSError, ValueError, KeyError):
                    return None
                self._memory_cache[key] = cfg
                return dict(cfg)
        return None

    def set(self, kernel_type: str, problem_size: Tuple[int, ...], device: str, config: Dict[str, Any]) -> None:
        key = self._make_key(kernel_type, problem_size, device)
        self._memory_cache[key] = dict(config)
        if self.cache_dir:
            payload = {"kernel_type": kernel_type, "problem_size": list(problem_size), "device": device,
                       "config": config}
            (self.cache_dir / f"{key}.json").write_text(json.dumps(payload, indent=2))

    def clear(self) -> None:
        self._memory_cache.clear()
        if self.cache_dir:
            for f in self.cache_dir.glob("*.json"):
                f.unlink()

    def get_all_keys(self) -> list:
        keys = set(self._memory_cache)
        if self.cache_dir:
            keys.update(f.stem for f in self.cache_dir.glob("*.json"))
        return sorted(keys)

    def __contains__(self, item: Tuple[str, Tuple[int, ...], str]) -> bool:
        return self.get(*item) is not None

    def __len__(self) -> int:
        return len(self.get_all_keys())

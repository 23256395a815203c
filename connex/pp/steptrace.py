"""Per-step timestamps for latency analysis (``CONNEX_PP_TRACE=1``;
reference ``connex/adapters/vllm/pp/trace.py``).

Each process appends ``<tag> <seq> <monotonic ns> <thread>`` lines to
``$CONNEX_PP_TRACE_DIR/cxtrace-<pid>.txt`` (default ``/dev/shm``), after a
``clock <wall ns> <monotonic ns> -`` anchor line.  CLOCK_MONOTONIC is one
clock for all processes of a host, so the files of a host's stages merge
into one timeline; the anchors align hosts to NTP accuracy.

``python -m connex.pp.steptrace FILE...`` (or ``connex.adapters.vllm.pp.trace``) merges files and prints,
per step (``seq``), every tag's offset from the step's first stamp (µs) and
the median per tag over all steps.
"""
from __future__ import annotations

import os
import statistics
import sys
import threading
import time
from collections import defaultdict
from typing import Dict, Iterable, List, Tuple

ON = os.getenv("CONNEX_PP_TRACE", "0") == "1"
_file = None
_lock = threading.Lock()


def tr(tag: str, seq: int) -> None:
    if not ON:
        return
    global _file
    t = time.monotonic_ns()
    with _lock:
        if _file is None:
            d = os.getenv("CONNEX_PP_TRACE_DIR", "/dev/shm")
            _file = open(os.path.join(d, f"cxtrace-{os.getpid()}.txt"), "a", buffering=1 << 16)
            _file.write(f"clock {time.time_ns()} {time.monotonic_ns()} -\n")
        _file.write(f"{tag} {seq} {t} {threading.current_thread().name}\n")


def flush() -> None:
    with _lock:
        if _file is not None:
            _file.flush()


def load(paths: Iterable[str]) -> List[Tuple[str, int, int]]:
    """``[(tag, seq, wall-aligned ns)]`` of all files, sorted by time."""
    out = []
    for p in paths:
        offset = 0
        with open(p) as f:
            for line in f:
                parts = line.split()
                if len(parts) < 3:
                    continue
                if parts[0] == "clock":
                    offset = int(parts[1]) - int(parts[2])
                    continue
                out.append((parts[0], int(parts[1]), int(parts[2]) + offset))
    return sorted(out, key=lambda r: r[2])


def timeline(records: List[Tuple[str, int, int]]) -> Dict[int, Dict[str, float]]:
    """Per step: tag -> µs after the step's first stamp (first stamp per tag)."""
    steps: Dict[int, Dict[str, int]] = defaultdict(dict)
    for tag, seq, t in records:
        steps[seq].setdefault(tag, t)
    return {s: {tag: (t - min(tags.values())) / 1e3 for tag, t in tags.items()} for s, tags in steps.items()}


def main(argv: List[str]) -> int:
    if not argv:
        print("usage: python -m connex.pp.steptrace cxtrace-*.txt", file=sys.stderr)
        return 2
    tl = timeline(load(argv))
    per_tag: Dict[str, List[float]] = defaultdict(list)
    for s in sorted(tl):
        row = sorted(tl[s].items(), key=lambda kv: kv[1])
        print(f"{s:#x} " + " ".join(f"{tag}=+{us:.1f}" for tag, us in row))
        for tag, us in row:
            per_tag[tag].append(us)
    print("median " + " ".join(f"{tag}=+{statistics.median(v):.1f}" for tag, v in
                                sorted(per_tag.items(), key=lambda kv: statistics.median(kv[1]))))
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))

"""Layer scheduler: the reference's ``src-code/scheduler.py`` API on this build.

``N730Scheduler(model_path, prefetch)`` keeps the reference's public surface
(``stream(start, end)``, ``get_layer(idx)``, ``stats``, ``print_stats()``,
``LayerBuffer``, ``SchedulerStats``; ``scheduler.py:108-311``) on top of this
repository's ``n730core`` C ABI (``include/n730core.h``): a background thread
reads + dequantises layers (per-tensor and group-wise blocks) into a bounded
queue while the caller consumes them.

The GPU side of layer streaming - weights held in pinned host memory and
copied into HBM slots ahead of the layer that needs them - lives in the C++
whole-model engine: ``n730_b200.engine.Engine(stream_depth=d)`` keeps every
layer's device image in pinned host memory and copies layer ``l + d`` into a
free HBM slot on a copy stream while layer ``l`` computes.
"""
from __future__ import annotations

import ctypes as C
import queue
import threading
import time
from dataclasses import dataclass
from pathlib import Path
from typing import Iterator, Optional

import numpy as np

from . import _lib
from .formats import read_header

N730_ERRORS = _lib.CORE_ERRORS


def check_err(code: int, context: str = ""):
    """Raise on a negative n730core return code (``scheduler.py:87-101``)."""
    if code < 0:
        raise RuntimeError(f"n730core error in {context}: {N730_ERRORS.get(code, f'unknown error {code}')}")


@dataclass
class LayerBuffer:
    layer_idx: int
    layer_name: str
    weights: np.ndarray      # float32 [rows, cols]
    precision: str
    load_time_ms: float      # read + dequant


@dataclass
class SchedulerStats:
    total_layers: int = 0
    total_bytes_read: int = 0
    total_load_ms: float = 0.0
    gpu_wait_ms: float = 0.0
    prefetch_hits: int = 0
    prefetch_misses: int = 0
    peak_ram_layers: int = 0

    @property
    def hit_rate(self) -> float:
        return self.prefetch_hits / max(self.prefetch_hits + self.prefetch_misses, 1)

    @property
    def avg_load_ms(self) -> float:
        return self.total_load_ms / max(self.total_layers, 1)

    @property
    def throughput_mb_s(self) -> float:
        return 0.0 if self.total_load_ms < 1 else (self.total_bytes_read / 2**20) / (self.total_load_ms / 1e3)


class N730Scheduler:
    """Read + dequantise ``.n730`` layers ahead of their use."""

    # a consumer that waited longer than this for a layer counts as a prefetch miss
    MISS_MS = 2.0

    def __init__(self, model_path: str, prefetch: int = 4, verbose: bool = True):
        self.model_path = Path(model_path)
        self.prefetch = prefetch
        self.stats = SchedulerStats()
        self._lib = _lib.core()
        self._handle = int(self._lib.n730_open(str(self.model_path).encode()))
        check_err(self._handle, "n730_open")
        self._header = read_header(self.model_path)
        self._seek_table = self._header["seek_table"]
        self._max_elements = max(e["rows"] * e["cols"] for e in self._seek_table)
        self._io = threading.Lock()  # the core handle is not safe for concurrent seeks
        if verbose:
            h = self._header
            print(f"  C++ core  : {self._lib.n730_version().decode()}")
            print(f"  Model     : {h.get('model_id', '?')}  layers {h.get('total_layers', len(self._seek_table))}"
                  f"  {h.get('stored_mb', '?')} MB ({h.get('compression', '?')}x)  prefetch {prefetch}")

    def close(self):
        if getattr(self, "_handle", 0) > 0:
            self._lib.n730_close(self._handle)
            self._handle = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _read_layer_cpp(self, entry: dict) -> LayerBuffer:
        out = np.empty(entry["rows"] * entry["cols"], np.float32)
        rows, cols, prec = C.c_int32(0), C.c_int32(0), C.c_int32(0)
        t0 = time.perf_counter()
        with self._io:
            rc = self._lib.n730_read_layer(self._handle, C.c_int64(entry["file_offset"]),
                                           out.ctypes.data_as(C.POINTER(C.c_float)),
                                           C.byref(rows), C.byref(cols), C.byref(prec))
        ms = (time.perf_counter() - t0) * 1e3
        check_err(rc, f"n730_read_layer (layer {entry['layer_idx']})")
        return LayerBuffer(entry["layer_idx"], entry["layer_name"], out.reshape(rows.value, cols.value),
                           entry["precision"], ms)

    def stream(self, start: int = 0, end: Optional[int] = None) -> Iterator[LayerBuffer]:
        """Yield layers [start, end) in file order, read by a background thread
        that stays at most ``prefetch + 1`` layers ahead."""
        end = len(self._seek_table) if end is None else end
        q: queue.Queue = queue.Queue(maxsize=self.prefetch + 1)
        failure = []

        def worker():
            try:
                for i in range(start, end):
                    e = self._seek_table[i]
                    layer = self._read_layer_cpp(e)
                    self.stats.total_layers += 1
                    self.stats.total_load_ms += layer.load_time_ms
                    self.stats.total_bytes_read += e["stored_bytes"]
                    q.put(layer)
                    self.stats.peak_ram_layers = max(self.stats.peak_ram_layers, q.qsize())
            except Exception as ex:  # surfaced to the consumer
                failure.append(ex)
            q.put(None)

        th = threading.Thread(target=worker, daemon=True)
        th.start()
        while True:
            t0 = time.perf_counter()
            layer = q.get()
            waited = (time.perf_counter() - t0) * 1e3
            if layer is None:
                break
            if waited < self.MISS_MS:
                self.stats.prefetch_hits += 1
            else:
                self.stats.prefetch_misses += 1
                self.stats.gpu_wait_ms += waited
            yield layer
        th.join()
        if failure:
            raise failure[0]

    def get_layer(self, layer_idx: int) -> LayerBuffer:
        """Random access to one layer (one seek + read + dequant)."""
        return self._read_layer_cpp(self._seek_table[layer_idx])

    def print_stats(self):
        s = self.stats
        print(f"  layers {s.total_layers}  read {s.total_bytes_read / 2**20:.1f} MB  avg {s.avg_load_ms:.2f} ms/layer"
              f"  {s.throughput_mb_s:.1f} MB/s  hit rate {s.hit_rate * 100:.1f}%  waited {s.gpu_wait_ms:.1f} ms"
              f"  peak queued {s.peak_ram_layers}")

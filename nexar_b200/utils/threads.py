"""Run one function per rank on threads (ranks of ``bootstrap_local`` live in
one process; each collective needs every rank to call it concurrently)."""
from __future__ import annotations

import threading
from typing import Callable, List, Sequence


def run_ranks(items: Sequence, fn: Callable, timeout: float = 120.0) -> List:
    """``fn(item)`` for every item on its own thread; results in item order.
    Re-raises the first exception; raises TimeoutError if a thread is still
    running after ``timeout`` seconds."""
    res = [None] * len(items)
    errs = [None] * len(items)

    def go(i):
        try:
            res[i] = fn(items[i])
        except BaseException as e:  # noqa: BLE001  (re-raised below on the caller's thread)
            errs[i] = e

    ts = [threading.Thread(target=go, args=(i,), daemon=True) for i in range(len(items))]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout)
        if t.is_alive():
            raise TimeoutError("a rank did not finish")
    for e in errs:
        if e is not None:
            raise e
    return res

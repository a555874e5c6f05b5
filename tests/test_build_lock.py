"""The library build is safe when several processes start it at once.

Every rank of a torchrun launch calls build() before it loads the library; if
a source is newer than the built library they must not compile over each
other.  The build takes an exclusive file lock and re-checks staleness under
it, so exactly one caller compiles.  Checked here with threads (each opens
the lock file separately, so the lock excludes them as it does processes) and
a stand-in for the compiler.
"""

from __future__ import annotations

import threading
import time

from local_kimi_b200 import build as build_mod


def test_concurrent_builds_compile_once(monkeypatch, tmp_path):
    state = {"stale": True, "active": 0, "max_active": 0, "compiles": 0}
    mu = threading.Lock()

    def fake_stale(target, inputs):
        return state["stale"]

    def fake_compile(srcs, headers, verbose, force, ptxas_verbose):
        with mu:
            state["active"] += 1
            state["max_active"] = max(state["max_active"], state["active"])
            state["compiles"] += 1
        time.sleep(0.2)
        with mu:
            state["stale"] = False
            state["active"] -= 1
        return build_mod.LIB_PATH

    monkeypatch.setattr(build_mod, "_stale", fake_stale)
    monkeypatch.setattr(build_mod, "_compile", fake_compile)
    monkeypatch.setattr(build_mod, "BUILD_DIR", tmp_path)
    results = []
    threads = [threading.Thread(target=lambda: results.append(build_mod.build())) for _ in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=30)
    assert len(results) == 4 and all(r == build_mod.LIB_PATH for r in results)
    assert state["compiles"] == 1
    assert state["max_active"] == 1

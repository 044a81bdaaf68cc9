"""The benchmark's workloads are the configurations the parity tests check.

``bench.py --workload cfg4`` packs configuration 4's documents with its own
copy of the length recipe (the benchmark must not import the tests); these
CPU tests keep it equal to the parity suite's ``cfg4_window_lengths``, and
check the mixer block's FLOP count against its GEMM shapes.
"""

from __future__ import annotations

import importlib.util
import os

from cases import cfg4_window_lengths

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_cfg4_boundaries_match_the_parity_recipe():
    bench = _bench()
    cu = bench.cfg4_cu_seqlens()
    ref = [0]
    for w in range(bench.CFG4_WINDOWS):
        for n in cfg4_window_lengths(w):
            ref.append(ref[-1] + n)
    assert cu == ref
    assert cu[-1] == bench.CFG4_WINDOWS * bench.T
    assert all(b > a for a, b in zip(cu, cu[1:]))
    # every window boundary is a document boundary
    assert all(w * bench.T in cu for w in range(bench.CFG4_WINDOWS + 1))


def test_mixer_flops_per_token():
    bench = _bench()
    inner = bench.H * bench.D
    gemm = 2 * (1536 * 4 * inner + 1536 * 128 + 128 * inner + 1536 * bench.H + inner * 1536)
    layer = sum(bench.KERNEL_FLOPS_PER_TOKEN_HEAD.values()) * bench.H
    assert bench.mixer_flops_per_token() == 3 * gemm + layer


def test_traffic_hash_covers_the_layer_kernels_headers():
    """The bench line says whether its DRAM traffic figures were captured on the
    kernels it times, by a hash of the headers the layer's five kernels are built
    from: every such header must be in the list (and exist), so that an edit to
    any of them marks the figures stale."""
    import re
    bench = _bench()
    csrc = os.path.join(ROOT, "sophia_b200", "csrc")
    listed = set(bench.LAYER_KERNEL_SOURCES)
    assert all(os.path.isfile(os.path.join(csrc, f)) for f in listed)
    # the include closure of the layer kernels' headers stays inside the list
    roots = {"kda_fwd.cuh", "kda_fwd_state_tc.cuh", "kda_bwd_state_tc.cuh", "kda_bwd_intra.cuh", "kda_post.cuh"}
    seen, todo = set(), list(roots)
    while todo:
        f = todo.pop()
        if f in seen:
            continue
        seen.add(f)
        with open(os.path.join(csrc, f)) as fh:
            todo += re.findall(r'#include "([^"/]+\.cuh)"', fh.read())
    assert seen <= listed, sorted(seen - listed)
    assert len(bench.kernel_source_hash()) == 16

"""chm_probe_noalloc (static device scratch, no allocation) against chm_probe
(caller workspace) through the C ABI: identical labels on two calls in a row,
and a clear capacity error beyond the static scratch.  Collected last so it
also runs after every other GPU test in the same process."""
import numpy as np
import pytest

from chimera_b200 import capi

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _unit_rows(rng, n):
    x = rng.standard_normal((n, 128)).astype(np.float32)
    return x / np.linalg.norm(x, axis=1, keepdims=True)


def _with_workspace(L, rows, cents, norms, nc, nprobe, stream):
    out = torch.full((rows.shape[0], nprobe), -1, dtype=torch.int32, device="cuda")
    nb = L.chm_probe_workspace_bytes(rows.shape[0], nc, nprobe)
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    capi.check(L.chm_probe(capi._ptr(rows), rows.shape[0], capi._ptr(cents), capi._ptr(norms), nc, nprobe,
                           capi._ptr(out), capi._ptr(ws), nb, stream), "chm_probe")
    return out


def _no_alloc(L, rows, cents, norms, nc, nprobe, stream):
    out = torch.full((rows.shape[0], nprobe), -1, dtype=torch.int32, device="cuda")
    capi.check(L.chm_probe_noalloc(capi._ptr(rows), rows.shape[0], capi._ptr(cents), capi._ptr(norms), nc,
                                   nprobe, capi._ptr(out), stream), "chm_probe_noalloc")
    return out


def test_probe_noalloc_matches_probe_twice():
    L = capi.lib()
    stream = capi._stream(torch)
    rng = np.random.default_rng(11)
    nc, nprobe = 20000, 128
    cents = torch.from_numpy(_unit_rows(rng, nc)).cuda()
    norms = torch.empty(nc, device="cuda")
    capi.check(L.chm_row_norms(capi._ptr(cents), nc, capi._ptr(norms), stream), "row_norms")
    for call in range(2):  # two calls in a row reuse the same static scratch
        rows = torch.from_numpy(_unit_rows(rng, 64 * (call + 1))).cuda()
        want = _with_workspace(L, rows, cents, norms, nc, nprobe, stream)
        got = _no_alloc(L, rows, cents, norms, nc, nprobe, stream)
        torch.cuda.synchronize()
        assert torch.equal(got, want), f"call {call}"
        assert int(got.min()) >= 0


def test_probe_noalloc_rejects_beyond_scratch():
    L = capi.lib()
    stream = capi._stream(torch)
    rng = np.random.default_rng(12)
    limit = capi.PROBE_NOALLOC_MAX_ELEMENTS
    rows_n = 32
    nc = limit // rows_n + 1  # one column past the scratch
    cents = torch.from_numpy(_unit_rows(rng, nc)).cuda()
    norms = torch.empty(nc, device="cuda")
    capi.check(L.chm_row_norms(capi._ptr(cents), nc, capi._ptr(norms), stream), "row_norms")
    rows = torch.from_numpy(_unit_rows(rng, rows_n)).cuda()
    out = torch.full((rows_n, 8), -1, dtype=torch.int32, device="cuda")
    st = L.chm_probe_noalloc(capi._ptr(rows), rows_n, capi._ptr(cents), capi._ptr(norms), nc, 8,
                             capi._ptr(out), stream)
    assert st == capi.CHM_ERR_CAPACITY
    assert b"exceeds the static scratch" in L.chm_last_error()
    torch.cuda.synchronize()
    assert int(out.max()) == -1  # nothing launched
    # at the limit itself it runs
    nc_ok = limit // rows_n
    got = _no_alloc(L, rows, cents[:nc_ok].contiguous(), norms[:nc_ok].contiguous(), nc_ok, 8, stream)
    want = _with_workspace(L, rows, cents[:nc_ok].contiguous(), norms[:nc_ok].contiguous(), nc_ok, 8, stream)
    torch.cuda.synchronize()
    assert torch.equal(got, want)

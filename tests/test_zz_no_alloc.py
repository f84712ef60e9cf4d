"""mgb_argmax_noalloc: greedy token choice without any device allocation.

Some callers cannot allocate device memory when they need a token picked: code
running inside another framework's stream capture, hosts whose caching
allocator already holds the GPU's memory, serving loops that forbid allocation.
This entry point keeps its scratch in a fixed static device array instead.

It is checked against the existing entry point mgb_greedy_logits, whose forced
token ids are the engine's fused argmax of the very logits it returns: two calls
in a row (sharing the static scratch) must give the same ids and maxima. The
file name makes pytest collect it last.
"""
import numpy as np
import pytest

from malaga_b200 import models

pytestmark = pytest.mark.gpu


def _entry():
    from malaga_b200 import _lib

    return _lib.load().mgb_argmax_noalloc  # typed by _lib.SIGNATURES


def test_argmax_noalloc_matches_greedy_ids_on_two_calls(gpu, model):
    import torch

    from malaga_b200 import Engine

    path = model("mid", "q4_k_m")
    V = models.config_of("mid").vocab_size
    src = models.random_sources(5, 3, 20, V, 3, src_tag=V - 1)
    eng = Engine(path)
    ids, logits = eng.greedy_logits(eng.encode(src), V - 2, 3, force=True)
    fn = _entry()
    rows = len(src)
    stream = torch.cuda.current_stream()
    for step in (0, 1):
        d_logits = torch.from_numpy(np.ascontiguousarray(logits[step])).cuda()
        d_ids = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
        d_vals = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
        rc = fn(d_logits.data_ptr(), rows, V, d_ids.data_ptr(), d_vals.data_ptr(), stream.cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        got = d_ids.cpu().numpy().view(np.uint32)
        np.testing.assert_array_equal(got, ids[:, step])
        np.testing.assert_array_equal(got, logits[step].argmax(axis=1))
        np.testing.assert_array_equal(d_vals.cpu().numpy(), logits[step].max(axis=1))


def test_argmax_noalloc_rejects_more_rows_than_its_scratch(gpu):
    import torch

    from malaga_b200 import _lib

    fn = _entry()
    x = torch.zeros((65, 8), dtype=torch.float32, device="cuda")
    out = torch.zeros(65, dtype=torch.int32, device="cuda")
    rc = fn(x.data_ptr(), 65, 8, out.data_ptr(), None, None)
    assert rc == _lib.MGB_ERR_INVALID
    assert b"64 rows" in _lib.load().mgb_last_error()


def test_argmax_noalloc_edge_rows(gpu):
    """64 rows (the warps of the second pass loop over rows) of 100 logits (most
    first-pass CTAs get an empty range), with a row of only -inf, a row whose
    maximum repeats (the lowest index wins, as numpy's argmax), and a row of only
    NaN (id 0): two calls in a row against numpy."""
    import torch

    rng = np.random.default_rng(5)
    x = rng.standard_normal((64, 100)).astype(np.float32)
    x[3, :] = -np.inf
    x[7, :] = 1.0
    x[7, [11, 40, 77]] = 2.5
    x[9, :] = np.nan
    want = x.argmax(axis=1)
    want[9] = 0
    fn = _entry()
    stream = torch.cuda.current_stream()
    for _ in range(2):
        d_x = torch.from_numpy(x).cuda()
        d_ids = torch.full((64,), -1, dtype=torch.int32, device="cuda")
        d_vals = torch.zeros(64, dtype=torch.float32, device="cuda")
        assert fn(d_x.data_ptr(), 64, 100, d_ids.data_ptr(), d_vals.data_ptr(), stream.cuda_stream) == 0
        torch.cuda.synchronize()
        got = d_ids.cpu().numpy()
        np.testing.assert_array_equal(got, want)
        vals = d_vals.cpu().numpy()
        ok = np.ones(64, bool)
        ok[9] = False
        np.testing.assert_array_equal(vals[ok], x[ok].max(axis=1))
        assert vals[9] == -np.inf and got[7] == 11 and got[3] == 0

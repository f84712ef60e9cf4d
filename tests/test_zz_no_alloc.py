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
import ctypes

import numpy as np
import pytest

from malaga_b200 import models

pytestmark = pytest.mark.gpu


def _entry():
    from malaga_b200 import _lib

    fn = _lib.load().mgb_argmax_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_void_p]
    return fn


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

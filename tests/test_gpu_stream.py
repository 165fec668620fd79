"""GPU: the diagnostic read stream (ps_stream_read) reads every byte exactly once.

Both methods (bulk asynchronous copies into shared memory, and 16-byte loads)
fold each 32-bit word into an XOR checksum; the test compares it with the same
XOR computed on the host, for sizes that do and do not fill a 32 KB chunk or the
unrolled grid stride, and checks that no wait bound ran out.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from paged_serve_b200 import _lib, ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.mark.parametrize("method", [_lib.PS_STREAM_BULK, _lib.PS_STREAM_LOADS])
@pytest.mark.parametrize("num_words", [4, 4 * 1000003, 8192 * 149 + 12, 4 * 148 * 256 * 8 * 3])
def test_checksum_covers_every_word_once(method, num_words):
    gen = torch.Generator().manual_seed(num_words)
    host = torch.randint(-2**31, 2**31 - 1, (num_words,), generator=gen, dtype=torch.int64)
    host = host.to(torch.int32)
    buf = host.to(DEV)
    acc = torch.zeros(1, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.stream_read(buf, acc, method, err)
    want = np.bitwise_xor.reduce(host.numpy().view(np.uint32))
    assert int(acc.cpu().numpy().view(np.uint32)[0]) == int(want)
    assert int(err.item()) == 0

"""GPU: the diagnostic read stream (ps_stream_read) reads every byte exactly once.

The kernel folds each 32-bit word into an XOR checksum; the test compares it
with the same XOR computed on the host, for sizes that do and do not fill the
unrolled grid stride, and for a capped grid.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from paged_serve_b200 import ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.mark.parametrize("num_words,ctas", [(4, 0), (4 * 1000003, 0), (4 * 333333, 5),
                                            (4 * 148 * 256 * 8 * 3, 0)])
def test_checksum_covers_every_word_once(num_words, ctas):
    gen = torch.Generator().manual_seed(num_words)
    host = torch.randint(-2**31, 2**31 - 1, (num_words,), generator=gen, dtype=torch.int64)
    host = host.to(torch.int32)
    buf = host.to(DEV)
    acc = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.stream_read(buf, acc, ctas)
    want = np.bitwise_xor.reduce(host.numpy().view(np.uint32))
    assert int(acc.cpu().numpy().view(np.uint32)[0]) == int(want)

"""The exponent exception tables compiled into the compressor equal torch's CPU
floor(log2(x)) on every normal binade, fp32 and bf16 (compressor.py:87)."""
import os
import re

import numpy as np
import torch

SRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                   "flashbfp_b200", "csrc", "log2_tables.h")


def _table(name):
    text = open(SRC).read()
    body = re.search(name + r"\[254\] = \{(.*?)\};", text, re.S).group(1)
    vals = [int(v) for v in re.findall(r"\d+", body)]
    assert len(vals) == 254
    return vals


def test_fp32_table_matches_torch():
    tab = _table("kLog2BumpF32")
    top = np.arange((1 << 23) - 64, 1 << 23, dtype=np.uint32)
    for e in range(-126, 128):
        x = torch.from_numpy((top + np.uint32((e + 127) << 23)).view(np.float32).copy())
        fl = torch.floor(torch.log2(x)).numpy()
        bumped = int((fl == e + 1).sum())
        assert bumped == min(tab[e + 126], 64), e
        assert np.all((fl == e) | (fl == e + 1))


def test_bf16_table_matches_torch():
    tab = _table("kLog2BumpBF16")
    for e in range(-126, 128):
        codes = (np.arange(128, dtype=np.uint32) + np.uint32((e + 127) << 7)).astype(np.uint16)
        x = torch.from_numpy(codes.view(np.int16).copy()).view(torch.bfloat16)
        fl = torch.floor(torch.log2(x)).float().numpy()
        assert int((fl == e + 1).sum()) == tab[e + 126], e
        # the bumped codes are exactly the top ones of the binade
        if tab[e + 126]:
            assert np.all(fl[128 - tab[e + 126]:] == e + 1)

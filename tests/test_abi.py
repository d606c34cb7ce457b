"""The C-ABI library loads on a CPU-only machine and exports what include/bolt3.h declares."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

from vsa_lm_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    txt = open(os.path.join(ROOT, "include", "bolt3.h")).read()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(bolt3_\w+)\s*\(", txt, re.M)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 8
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/bolt3.h but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"
    assert lib.bolt3_abi_version() == _lib.ABI_VERSION == 10
    assert lib.bolt3_status_string(0) == b"ok"
    assert b"shape" in lib.bolt3_status_string(2)


def test_struct_sizes_are_c_layout():
    # the ctypes mirrors have the compiled structs' sizes (a field added on one side only shows here)
    lib = _lib.load()
    for i, st in enumerate((_lib.PrepArgs, _lib.ConsolidateArgs, _lib.AttendArgs, _lib.PrefillArgs, _lib.AnchorArgs,
                            _lib.RMSNormArgs, _lib.SiluMulArgs)):
        assert ctypes.sizeof(st) % 8 == 0
        assert lib.bolt3_args_size(i) == ctypes.sizeof(st), st.__name__
    assert lib.bolt3_args_size(7) == 0


def test_entry_points_reject_bad_arguments_without_a_gpu():
    lib = _lib.load()
    assert lib.bolt3_prep(None, None) == 1
    assert lib.bolt3_consolidate(None, None) == 1
    assert lib.bolt3_attend(None, None) == 1
    assert lib.bolt3_prefill_fwd(None, None) == 1
    assert lib.bolt3_anchor_decode(None, None) == 1
    assert lib.bolt3_rmsnorm(None, None) == 1
    assert lib.bolt3_silu_mul(None, None) == 1
    sm = _lib.SiluMulArgs(gu=16, y=32, rows=4, I=100)
    assert lib.bolt3_silu_mul(ctypes.byref(sm), None) == 2         # I not a multiple of 8
    rn = _lib.RMSNormArgs(x=16, w=32, y=48, rows=4, x_stride=100, D=100, eps=1e-6)
    assert lib.bolt3_rmsnorm(ctypes.byref(rn), None) == 2          # D not a multiple of 8
    rn.D, rn.x_stride, rn.y = 128, 128, 40
    assert lib.bolt3_rmsnorm(ctypes.byref(rn), None) == 3          # misaligned output
    an = _lib.AnchorArgs(B=2, H=8, HKV=2, HD=128, q=16, k_new=32, v_new=48, k_cache=64, v_cache=80, cap=10, n=10,
                         y=96, scale=0.1)
    assert lib.bolt3_anchor_decode(ctypes.byref(an), None) == 4    # no room for the appended token
    an.n, an.HD = 3, 96
    assert lib.bolt3_anchor_decode(ctypes.byref(an), None) == 2    # unsupported head dim
    an.HD, an.q = 128, 8
    assert lib.bolt3_anchor_decode(ctypes.byref(an), None) == 3    # misaligned query rows
    an.q, an.pos_dev, an.pos_ref, an.pos_span = 16, 112, 3, 8
    assert lib.bolt3_anchor_decode(ctypes.byref(an), None) == 4    # 3 + 7 + 1 > 10
    a = _lib.ConsolidateArgs()
    assert lib.bolt3_consolidate(ctypes.byref(a), None) == 1      # null state pointers
    assert lib.bolt3_prefill_workspace_size(4, 1024, 96) == 0      # unsupported head dim


def test_prep_validates_parts_and_columns_without_a_gpu():
    """Fake (never dereferenced) 16-byte-aligned addresses: every case returns before a launch."""
    lib = _lib.load()
    fake = 1 << 20

    def args(**kw):
        a = _lib.PrepArgs(proj=fake, ld=1024, B=1, T=4, H=4, HKV=2, HD=64, inv_freq=fake, eps=1e-6,
                          q_raw=fake, q_rope=fake, eta=fake, k_raw=fake, k_rope=fake, v=fake, beta=fake,
                          q_head_stride=4, k_head_stride=4, eta_head_stride=4, beta_head_stride=4, parts=2,
                          k_col=0, v_col=128, beta_col=256)
        for k, v in kw.items():
            setattr(a, k, v)
        return lib.bolt3_prep(ctypes.byref(a), None)

    assert args(parts=0) == 1 and args(parts=4) == 1                  # BOLT3_ERR_ARG
    assert args(k_raw=0) == 1                                         # k/v/beta outputs required
    assert args(parts=1, q_col=0, eta_col=1020, q_raw=0) == 1         # q/eta outputs required
    cap = 4                                                           # BOLT3_ERR_CAPACITY
    assert args(v_col=1000) == cap                                    # section runs past the row
    assert args(k_col=4) == 3                                         # BOLT3_ERR_ALIGN: section start
    assert args(parts=1, q_col=0, eta_col=1022) == cap                # eta logits past the row
    assert args(k_head_stride=3) == cap                               # T does not fit the buffer
    assert args(ld=1020) == 3                                         # BOLT3_ERR_ALIGN: row stride


def test_workspace_size_formula():
    lib = _lib.load()
    # T = 1024: 8 chunks -> 6 consolidations; per chain-snapshot: 2*S*HD*2 + S*4 + S + HD*HD*4
    n = lib.bolt3_prefill_workspace_size(5, 1024, 64)
    per = 2 * 128 * 64 * 2 + 128 * 4 + 128 + 64 * 64 * 4
    assert per * 5 * 6 <= n <= per * 5 * 6 + 5 * 256
    assert lib.bolt3_prefill_workspace_size(5, 256, 64) <= 5 * 256   # no consolidation at T = 2C


def _emulated(vals, k, largest):
    lib = _lib.load()
    v = np.ascontiguousarray(vals, dtype=np.float32)
    out = np.zeros(k, dtype=np.int32)
    bad = lib.bolt3_topk_order_host(v.ctypes.data, len(v), k, int(largest), out.ctypes.data)
    assert bad == 0
    return out


@pytest.mark.parametrize("seed", range(4))
def test_topk_tie_order_matches_torch_cpu(seed):
    """The kernels' tie-order emulation reproduces CPU torch.topk exactly, ties and NaNs included."""
    g = torch.Generator().manual_seed(seed)
    for trial in range(1500):
        n = int(torch.randint(1, 260, (1,), generator=g))
        if trial % 3 == 0:
            n = 128
        k = n if trial % 4 == 0 else int(torch.randint(1, n + 1, (1,), generator=g))
        levels = int(torch.randint(1, 9, (1,), generator=g))
        x = torch.randint(0, levels, (n,), generator=g).float() * 0.125
        if trial % 7 == 0:
            x = torch.rand(n, generator=g)
        if trial % 13 == 0:
            x[torch.rand(n, generator=g) < 0.1] = float("nan")
        largest = bool(trial % 2)
        ref = torch.topk(x, k, largest=largest).indices.numpy()
        got = _emulated(x.numpy(), k, largest)
        assert np.array_equal(ref, got), (n, k, largest, x.tolist())

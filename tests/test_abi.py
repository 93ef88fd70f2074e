"""The C ABI library on CPU: it loads, exports every symbol include/b2pa.h
declares, and rejects bad arguments with status codes before touching the
GPU.  No kernel runs here."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from b2pa import _lib

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "b2pa.h"


def _declared() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"B2PA_API\s+[\w\s\*]+?\b(b2pa_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not _lib.LIB_PATH.exists():
        import __graft_entry__  # noqa: F401  (repo root on sys.path)

        __graft_entry__.build()
    return _lib.load()


def test_header_declares_the_abi():
    names = _declared()
    assert "b2pa_paged_decode" in names and "b2pa_kv_append" in names and "b2pa_paged_prefill" in names
    assert len(names) >= 10


def test_every_declared_symbol_is_exported_and_bound(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (b2pa_\w+)", out))
    for name in _declared():
        assert name in exported, f"{name} declared in b2pa.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes binding"
        assert getattr(lib, name) is not None


def test_abi_version(lib):
    m = re.search(r"#define B2PA_ABI_VERSION (\d+)", HEADER.read_text())
    assert lib.b2pa_abi_version() == int(m.group(1))


def test_status_codes_match_header():
    text = HEADER.read_text()
    for code, name in _lib.STATUS_NAMES.items():
        assert re.search(rf"{name}\s*=\s*{code}\b", text), name


def _decode(lib, **kw):
    args = dict(q=4096, qs=(64, 64, 64, 1), kp=16, vp=16, ps=(16 * 64, 16 * 64, 64, 1), nb=10, pt=8, pts=4,
                mp=4, sl=8, cl=8, out=8192, os=(64, 64, 64, 1), B=1, H=1, D=64, bs=16, dt=0, ws=256, wsb=1 << 30)
    args.update(kw)
    i64 = lambda t: (ctypes.c_int64 * 4)(*t)
    return lib.b2pa_paged_decode(args["q"], i64(args["qs"]), args["kp"], args["vp"], i64(args["ps"]), args["nb"],
                                 args["pt"], args["pts"], args["mp"], args["sl"], args["cl"], args["out"],
                                 i64(args["os"]), args["B"], args["H"], args["D"], args["bs"], 0.125, args["dt"],
                                 args["ws"], args["wsb"], None, None)


def test_decode_argument_validation(lib):
    assert _decode(lib, H=0) == -1
    assert _decode(lib, dt=7) == -2
    assert _decode(lib, D=48, ps=(16 * 48, 16 * 48, 48, 1)) == -2
    assert _decode(lib, bs=12) == -2
    assert _decode(lib, ps=(1, 16 * 64, 64, 1)) == -2            # pools not contiguous
    assert _decode(lib, qs=(64, 64, 64, 2)) == -2                # non-unit D stride
    assert _decode(lib, q=0) == -1                               # null q
    assert _decode(lib, pts=2) == -1                             # row stride < max_pages
    assert _decode(lib, wsb=16) == -4                            # workspace too small
    assert _decode(lib, ws=0) == -4                              # missing workspace
    assert _decode(lib, B=0) == 0                                # empty batch: nothing to do
    assert "workspace" in _lib.last_error() or _lib.last_error() == ""


def _decode_append(lib, **kw):
    args = dict(q=4096, qs=(64, 64, 64, 1), kn=8192, ks=(64, 64, 64, 1), vn=12288, vs=(64, 64, 64, 1), kp=16, vp=16,
                ps=(16 * 64, 16 * 64, 64, 1), nb=10, pt=8, pts=4, mp=4, sl=8, cl=8, st=8, ln=8, so=0, out=8192,
                os=(64, 64, 64, 1), B=1, H=1, D=64, bs=16, dt=0, ws=256, wsb=1 << 30)
    args.update(kw)
    i64 = lambda t: (ctypes.c_int64 * 4)(*t)
    return lib.b2pa_paged_decode_append(
        args["q"], i64(args["qs"]), args["kn"], i64(args["ks"]), args["vn"], i64(args["vs"]), args["kp"], args["vp"],
        i64(args["ps"]), args["nb"], args["pt"], args["pts"], args["mp"], args["sl"], args["cl"], args["st"],
        args["ln"], args["so"] or None, args["out"], i64(args["os"]), args["B"], args["H"], args["D"], args["bs"],
        0.125, args["dt"], args["ws"], args["wsb"], None, None)


def test_decode_append_argument_validation(lib):
    """b2pa_paged_decode_append rejects bad arguments before launching."""
    assert _decode_append(lib, H=0) == -1
    assert _decode_append(lib, dt=7) == -2
    assert _decode_append(lib, kn=0) == -1                           # null k_new
    assert _decode_append(lib, st=0) == -1                           # null start positions
    assert _decode_append(lib, ks=(64, 64, 64, 2)) == -2             # non-unit head_dim stride
    assert _decode_append(lib, vn=12290) == -2                       # new V rows not 4-byte aligned
    assert _decode_append(lib, ps=(1, 16 * 64, 64, 1)) == -2         # pools not contiguous
    assert _decode_append(lib, wsb=16) == -4                         # workspace too small
    assert _decode_append(lib, B=0) == 0                             # empty batch: nothing to do


def test_prefill_append_argument_validation(lib):
    """b2pa_paged_prefill_append rejects bad arguments before launching."""
    i64 = lambda t: (ctypes.c_int64 * 4)(*t)
    B, H, T, D, bs, mp = 1, 1, 8, 64, 16, 4
    qs = (T * H * D, D, H * D, 1)

    def call(kn=8192, ks=qs, st=8, T=T, dt=0):
        return lib.b2pa_paged_prefill_append(4096, i64(qs), kn, i64(ks), 12288, i64(qs), 16, 16,
                                             i64((H * bs * D, bs * D, D, 1)), 10, 8, mp, mp, 8, 8, st, 8, None,
                                             8192, i64(qs), B, H, T, D, bs, 0.125, dt, 256, 1 << 30, None, None)

    assert call(kn=0) == -1                      # null k_new
    assert call(st=0) == -1                      # null start positions
    assert call(ks=(T * H * D, D, H * D, 2)) == -2  # non-unit head_dim stride
    assert call(dt=7) == -2
    assert call(T=0) == 0                        # empty chunk: nothing to do


def test_prefill_f32_split_needs_its_workspace(lib):
    """fp32 head_dim 64 prefill runs on split copies of the pages held in the
    workspace: a missing or short workspace is refused before any launch."""
    i64 = lambda t: (ctypes.c_int64 * 4)(*t)
    B, H, T, D, bs, mp = 2, 2, 8, 64, 16, 4
    need = lib.b2pa_paged_prefill_workspace_size(B, H, T, D, mp, bs, 0)
    assert need > 0
    qs = (T * H * D, D, H * D, 1)
    args = [4096, i64(qs), 16, 16, i64((H * bs * D, bs * D, D, 1)), 10, 8, mp, mp, 8, 8, 8192, i64(qs),
            B, H, T, D, bs, 0.125, 0]
    assert lib.b2pa_paged_prefill(*args, None, 0, None, None) == -4
    assert lib.b2pa_paged_prefill(*args, 256, need - 256, None, None) == -4
    assert "workspace" in _lib.last_error()


def test_workspace_size_is_monotone(lib):
    f = lib.b2pa_paged_decode_workspace_size
    a = f(64, 8, 64, 65, 16, 0)
    b = f(64, 8, 64, 130, 16, 0)
    c = f(512, 32, 128, 513, 16, 1)
    assert 0 < a <= b
    assert c > 0 and c % 256 == 0
    assert f(0, 8, 64, 65, 16, 0) == 0
    # 4096 head-group streams (config[4]): the contiguous split keeps two
    # partial slots per CTA slot, whatever the context length; so do 512
    # streams, while 256 take the item split (partials grow with the length)
    assert f(512, 32, 128, 1026, 16, 1) == c
    assert c < 8 << 20
    assert f(64, 32, 128, 4096, 16, 1) < 8 << 20
    assert f(32, 32, 128, 4096, 16, 1) > 32 << 20
    # fp32, head_dim 64 (tensor cores on fp16 hi/lo splits): the split copies
    # of K and V (B * max_pages slots x H pages x block x 2D halves) + the slot table
    n = lib.b2pa_paged_prefill_workspace_size(8, 8, 256, 64, 32, 16, 0)
    assert n >= 2 * (8 * 32) * 8 * 16 * (2 * 64) * 2 + 4 * 8 * 32 and n % 256 == 0
    assert lib.b2pa_paged_prefill_workspace_size(8, 8, 256, 64, 0, 16, 0) == 0      # no pages: no copy
    # fp32, head_dim 128 (register-tiled path): at most 8 key tiles (512 keys) per CTA
    assert lib.b2pa_paged_prefill_workspace_size(8, 8, 256, 128, 32, 16, 0) == 0    # 512 keys: no split
    n = lib.b2pa_paged_prefill_workspace_size(8, 8, 256, 128, 64, 16, 0)            # 1024 keys: 2 splits
    assert n >= 8 * 8 * 256 * 2 * (128 + 2) * 4 and n % 256 == 0
    assert lib.b2pa_paged_prefill_workspace_size(8, 8, 256, 32, 64, 16, 0) == 0     # head_dim 32: general kernel
    assert lib.b2pa_paged_prefill_workspace_size(8, 8, 256, 64, 65, 16, 1) == 0  # bf16 config[2]: one wave, no split
    assert lib.b2pa_paged_prefill_workspace_size(1, 8, 256, 64, 65, 16, 1) > 0   # one sequence: key-range split


def test_append_and_zero_argument_validation(lib):
    i64 = lambda t: (ctypes.c_int64 * 4)(*t)
    ok = (256, 64, 64, 1)
    pool = (8 * 16 * 64, 16 * 64, 64, 1)
    rc = lib.b2pa_kv_append(8, i64(ok), 8, i64(ok), 16, 16, i64((1, 1, 1, 1)), 10, 8, 4, 4, 8, 8, 1, 8, 1, 64, 16, 0,
                            None, None)
    assert rc == -2
    rc = lib.b2pa_kv_append(8, i64(ok), 8, i64(ok), 16, 16, i64(pool), 10, 8, 4, 4, 8, 8, 1, 8, 1, 64, 16, 9, None, None)
    assert rc == -2
    rc = lib.b2pa_kv_append(8, i64(ok), 8, i64(ok), 16, 16, i64(pool), 10, 8, 4, 4, 8, 8, 0, 8, 1, 64, 16, 0, None, None)
    assert rc == 0
    assert lib.b2pa_zero_blocks(16, 16, i64(pool), 10, 8, -1, 8, 64, 16, 0, None, None) == -1
    assert lib.b2pa_zero_blocks(16, 16, i64(pool), 10, 8, 0, 8, 64, 16, 0, None, None) == 0


def test_missing_library_raises(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setenv("B2PA_LIB", str(tmp_path / "nope.so"))
    with pytest.raises(RuntimeError, match="not found"):
        _lib.load()


def test_row_ops_argument_validation(lib):
    """The decode-step row operations refuse bad arguments before launching
    (addresses are never dereferenced here)."""
    def linear(M=2, K=64, N=32, x=4096, xs=64, w=1 << 20, y=1 << 22, ys=32, act=0, ln=None):
        return lib.b2pa_rows_linear(x, xs, M, K, ln, None, 1e-5, w, None, N, act, y, ys, 0, None, None)

    assert linear(M=17) == -1                      # more than 16 rows
    assert linear(K=62, xs=64) == -2               # K not a multiple of 4
    assert linear(xs=60) == -2                     # row stride below K
    assert linear(x=4100) == -2                    # x not 16-byte aligned
    assert linear(act=3) == -2                     # unknown activation
    assert linear(ln=4104) == -2                   # LayerNorm weight not 16-byte aligned
    assert linear(y=4096 + 256) == -1              # y overlaps x
    assert "overlaps" in _lib.last_error()
    assert linear(M=0) == 0                        # nothing to do
    assert lib.b2pa_rows_embed(None, None, 1, 16, 10, 16, 10, 64, 16, 64, None, None) == -1
    assert lib.b2pa_rows_embed(16, 16, 1, 16, 10, 16, 10, 62, 16, 64, None, None) == -2
    assert lib.b2pa_rows_argmax(16, 10, 1, 20, 16, None, None) == -1  # row stride below N
    assert lib.b2pa_rows_argmax(16, 20, 0, 20, 16, None, None) == 0

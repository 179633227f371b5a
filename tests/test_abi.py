"""The C-ABI library loads and exports every symbol include/vlb200.h declares; host-side logic
that needs no GPU. (No compute call is made here.)"""

import re
from pathlib import Path

import numpy as np
import pytest

import vastloom_b200 as vb
from vastloom_b200 import synth

HEADER = Path(__file__).resolve().parent.parent / "include" / "vlb200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(vlb_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = vb.load_library()
    declared = declared_functions()
    assert len(declared) >= 25
    for name in declared:
        assert hasattr(lib, name), name
    assert sorted(vb.EXPORTS) == declared


def test_abi_version_and_status_mapping():
    lib = vb.load_library()
    assert lib.vlb_abi_version() == 2
    # ErrorCode order of include/vastloom/core/status.hpp:10-21, shifted by one
    assert [vb.ERROR_CODES[i] for i in range(1, 11)] == [
        "invalid_argument", "invalid_format", "not_found", "permission_denied", "io_error",
        "integrity_error", "unsafe_path", "unsupported", "resource_exhausted", "internal_error"]


def test_null_handle_is_an_error_not_a_crash():
    import ctypes as C

    lib = vb.load_library()
    buf = C.create_string_buffer(64)
    assert lib.vlb_synchronize(None) == 1
    assert lib.vlb_last_error(None, buf, 64) == 0
    assert b"null handle" in buf.value


def test_block_layouts_and_matrix_bytes():
    assert vb.matrix_bytes(vb.TYPE_IQ2_XXS, 2048, 4096) == 2_162_688
    assert vb.matrix_bytes(vb.TYPE_Q8_0, 2048, 4096) == 8_912_896
    assert vb.matrix_bytes(vb.TYPE_IQ1_S, 2048, 4096) == 1_638_400
    assert vb.matrix_bytes(vb.TYPE_IQ3_XXS, 4096, 2048) == 3_211_264
    assert vb.matrix_bytes(vb.TYPE_Q4_K, 2048, 4096) == 2048 * 16 * 144
    assert vb.matrix_bytes(vb.TYPE_Q6_K, 2048, 4096) == 2048 * 16 * 210
    assert vb.matrix_bytes(vb.TYPE_MXFP4, 2048, 4096) == 2048 * 128 * 17
    with pytest.raises(ValueError):
        vb.matrix_bytes(vb.TYPE_IQ2_XXS, 1, 100)


def test_synthetic_blocks_follow_the_configuration():
    rng = np.random.default_rng(0)
    for t in (vb.TYPE_Q8_0, vb.TYPE_IQ2_XXS, vb.TYPE_IQ3_XXS, vb.TYPE_IQ1_S, vb.TYPE_Q4_K, vb.TYPE_Q5_K,
              vb.TYPE_Q6_K, vb.TYPE_IQ2_S):
        be, bb = vb.BLOCK_LAYOUT[t]
        b = synth.blocks(rng, t, 100, 0.01).reshape(100, bb)
        at = 208 if t == vb.TYPE_Q6_K else 0  # the fp16 block scale
        d = (b[:, at].astype(np.uint16) | (b[:, at + 1].astype(np.uint16) << 8)).view(np.float16)
        assert np.all(np.isfinite(d)) and np.all(d >= 0)
        if t == vb.TYPE_Q8_0:
            q = b[:, 2:].view(np.int8)
            assert q.min() >= -127 and q.max() <= 127


def test_synthetic_zipf_logits_are_skewed():
    spec = synth.config(4, "small")
    _, _, logits = synth.activations(spec, 2000, seed=1)
    top1 = np.argmax(logits, axis=1)
    counts = np.bincount(top1, minlength=spec.experts)
    assert counts.max() > 4 * counts.mean()


def test_hash_tables_have_distinct_experts_per_row():
    spec = synth.config(2, "small")
    W = synth.layer_weights(spec, seed=3)
    t = W.tid2eid
    assert t.shape == (spec.vocab, 6)
    assert all(len(set(row)) == 6 for row in t[:200].tolist())


def test_codebook_file_roundtrip(grids):
    assert set(grids) == {16, 18, 19, 22}
    assert len(grids[19]) == 2048 * 8 and len(grids[16]) == 256 * 8 and len(grids[18]) == 256 * 4
    assert len(grids[22]) == 1024 * 8


def test_ep_driver_reports_the_nccl_it_binds():
    """The expert-parallel driver loads NCCL at first use (after torch, whose copy it then binds)
    and needs >= 2.18; no GPU is touched."""
    import ctypes as C

    import torch  # noqa: F401

    lib = vb.load_library()
    v = C.c_int(0)
    st = lib.vlb_ep_nccl_version(C.byref(v))
    if st == 8:  # VLB_ERR_UNSUPPORTED: no NCCL in this environment
        pytest.skip("no NCCL library")
    assert st == 0 and v.value >= 21800
    buf = C.create_string_buffer(128)
    assert lib.vlb_ep_comm_init(None, None, 0, 1, 1000, None) == 1  # invalid argument, not a crash
    assert lib.vlb_ep_forward_device(None, None, None, None, 0, None, None) == 1
    assert lib.vlb_ep_last_phases(None, None, None) == 1

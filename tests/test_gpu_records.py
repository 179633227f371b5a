"""Expert records to device (vlb_upload_record_async): one expert's ggml bytes, as an expert pack
holds them (deepseek_v4_expert_pack.hpp:24-41), go to the device in one copy and are re-laid out
there. Every matrix must come out identical to the host-path upload (vlb_upload_matrix): same
dequantized bits, same matvec bits, same layer outputs; the block checks must reject exactly what
the reference's decoders reject; the governor hooks are charged only above the caller's
reservation (ResidencyObject::begin_vram_copy, residency.cpp:183-198)."""

import time

import numpy as np
import pytest

import vastloom_b200 as vb
from vastloom_b200 import synth

pytestmark = pytest.mark.gpu

ALL_TYPES = [8, 16, 18, 19, 12, 13, 14, 22, 39]


def _record(rng, types_shapes, lead=5):
    """A record of ggml tensors behind `lead` junk bytes (odd offsets)."""
    parts = [rng.integers(0, 256, lead, dtype=np.uint8)]
    tensors, off = [], lead
    for i, (t, rows, cols) in enumerate(types_shapes):
        b = np.asarray(synth.matrix(rng, t, rows, cols, synth.D_SCALE[t]), np.uint8).reshape(-1)
        parts.append(b)
        tensors.append((0x5000 + 2 * i + 1, t, rows, cols, off, b.nbytes))
        off += b.nbytes
    return np.concatenate(parts), tensors


def _same_as_host_path(device, rec, tensors, mats):
    for m, (ident, t, rows, cols, off, nb) in zip(mats, tensors):
        ref = device.upload_matrix(t, rows, cols, rec[off:off + nb], identity=ident)
        try:
            assert vb.load_library().vlb_matrix_bytes(m.ptr) == vb.load_library().vlb_matrix_bytes(ref.ptr)
            a, b = device.dequantize(m), device.dequantize(ref)
            assert a.view(np.uint32).tobytes() == b.view(np.uint32).tobytes()
            x = np.random.default_rng(cols).standard_normal(cols).astype(np.float32)
            assert device.matvec(m, x).tobytes() == device.matvec(ref, x).tobytes()
        finally:
            device.release_matrix(ref)


@pytest.mark.parametrize("t", ALL_TYPES)
def test_gpu_record_matches_host_upload(device, t):
    rng = np.random.default_rng(100 + t)
    H, I = 512, 256
    rec, tensors = _record(rng, [(t, I, H), (t, I, H), (t, H, I)])
    mats = device.upload_record(rec, tensors).finish()
    try:
        _same_as_host_path(device, rec, tensors, mats)
    finally:
        for m in mats:
            device.release_matrix(m)


def test_gpu_record_full_size_expert_from_pinned_memory(device):
    """A config-2 expert (IQ1_S gate/up 2048 x 4096, IQ3_XXS down 4096 x 2048: 6.5 MB) from
    page-locked memory; several records in flight at once."""
    rng = np.random.default_rng(7)
    shapes = [(vb.TYPE_IQ1_S, 2048, 4096), (vb.TYPE_IQ1_S, 2048, 4096), (vb.TYPE_IQ3_XXS, 4096, 2048)]
    recs = [_record(rng, shapes, lead=0) for _ in range(3)]
    pins, ups = [], []
    try:
        for rec, tensors in recs:
            pin = device.host_buffer(rec.nbytes)
            pin.array[:] = rec
            pins.append(pin)
            ups.append(device.upload_record(pin.array, tensors))
        t0 = time.time()
        while not ups[-1].done():
            assert time.time() - t0 < 30.0
            time.sleep(0.001)
        for (rec, tensors), up in zip(recs, ups):
            mats = up.finish()
            try:
                _same_as_host_path(device, rec, tensors, mats)
            finally:
                for m in mats:
                    device.release_matrix(m)
    finally:
        for pin in pins:
            pin.free()


def test_gpu_record_rejects_what_the_reference_rejects(device):
    rng = np.random.default_rng(11)
    shapes = [(vb.TYPE_IQ2_XXS, 256, 512), (vb.TYPE_Q8_0, 256, 512), (vb.TYPE_IQ3_XXS, 512, 256)]
    rec, tensors = _record(rng, shapes)
    for m in device.upload_record(rec, tensors).finish():  # grows the staging copy first
        device.release_matrix(m)
    before = device.allocated_bytes()
    bad = rec.copy()
    off = tensors[1][4] + 7 * 34  # Q8_0 block 7 of tensor 1: d = +inf
    bad[off:off + 2] = [0x00, 0x7C]
    with pytest.raises(vb.VlbError) as e:
        device.upload_record(bad, tensors).finish()
    assert e.value.code == "invalid_format" and "record tensor 1" in str(e.value)
    assert device.allocated_bytes() == before
    with pytest.raises(vb.VlbError) as e:
        device.upload_matrix(vb.TYPE_Q8_0, 256, 512, bad[off - 7 * 34:off - 7 * 34 + tensors[1][5]])
    assert e.value.code == "invalid_format"
    # argument checks happen before anything is enqueued
    t0 = list(tensors[0])
    with pytest.raises(vb.VlbError) as e:
        device.upload_record(rec[:tensors[2][4]], tensors)
    assert e.value.code == "invalid_format"
    with pytest.raises(vb.VlbError) as e:
        device.upload_record(rec, [tuple(t0[:5] + [t0[5] - 66])])
    assert e.value.code == "invalid_format"
    with pytest.raises(vb.VlbError) as e:
        device.upload_record(rec, [tuple([t0[0], 10] + t0[2:])])
    assert e.value.code == "unsupported"
    assert device.allocated_bytes() == before


def test_gpu_record_mxfp4_finite_rule_matches_host_path(device):
    """MXFP4 blocks at the top of the E8M0 range: the record path and the host path accept and
    reject the same blocks (a value of at least 2^128 is not finite)."""
    for e in (252, 253, 254, 255):
        for code in range(8):
            blk = np.zeros((32, 17), np.uint8)
            blk[:, 0] = 127
            blk[5, 0] = e
            blk[5, 3] = code | (1 << 4)
            payload = blk.reshape(-1)
            outcomes = []
            for path in ("host", "record"):
                try:
                    if path == "host":
                        m = device.upload_matrix(vb.TYPE_MXFP4, 32, 32, payload)
                    else:
                        (m,) = device.upload_record(payload, [(3, vb.TYPE_MXFP4, 32, 32, 0, payload.nbytes)]).finish()
                    device.release_matrix(m)
                    outcomes.append(True)
                except vb.VlbError as err:
                    assert err.code == "invalid_format"
                    outcomes.append(False)
            mags = [0, 1, 2, 3, 4, 6, 8, 12]
            finite = max(mags[code], 1) * 2.0 ** (e - 128) < 2.0 ** 128
            assert outcomes == [finite, finite], (e, code)


def test_gpu_record_governor_charges_only_above_the_reservation():
    class Gov:
        def __init__(self):
            self.used = 0

        def reserve(self, n, tag):
            self.used += n
            return True

        def release(self, n, tag):
            self.used -= n

    gov = Gov()
    rng = np.random.default_rng(3)
    rec, tensors = _record(rng, [(vb.TYPE_IQ2_XXS, 256, 1024), (vb.TYPE_IQ2_XXS, 256, 1024),
                                 (vb.TYPE_IQ2_XXS, 1024, 256)], lead=0)
    with vb.Device(0, governor=gov) as dev:
        for m in dev.upload_record(rec, tensors).finish():
            dev.release_matrix(m)
        base_gov, base_alloc = gov.used, dev.allocated_bytes()
        mats = dev.upload_record(rec, tensors, reserved_bytes=rec.nbytes).finish()
        images = dev.allocated_bytes() - base_alloc
        assert images > rec.nbytes  # split scales and tile padding cost a little more than the payload
        assert gov.used - base_gov == images - rec.nbytes
        for m in mats:
            dev.release_matrix(m)
        assert gov.used == base_gov and dev.allocated_bytes() == base_alloc
        # a reservation larger than the images: nothing is charged
        mats = dev.upload_record(rec, tensors, reserved_bytes=10 * rec.nbytes).finish()
        assert gov.used == base_gov
        for m in mats:
            dev.release_matrix(m)
        assert gov.used == base_gov


@pytest.mark.parametrize("cfg", [1, 2, 3])
def test_gpu_layer_from_records_is_bit_identical(device, cfg):
    spec = synth.config(cfg, "small")
    W = synth.layer_weights(spec, seed=40 + cfg)
    x, tok, logits = synth.activations(spec, 64, seed=41)
    outs = []
    for records in (False, True):
        layer = synth.upload_layer(device, W, max_tokens=64, records=records)
        try:
            runs = [layer.forward(x[:4], None if tok is None else tok[:4], None if logits is None else logits[:4])]
            if cfg == 3:
                layer.set_prefill_tokens(1)
            runs.append(layer.forward(x, tok, logits))
            outs.append(runs)
        finally:
            layer.destroy()
            for lst in layer.matrices.values():
                for m in lst:
                    device.release_matrix(m)
            for m in layer.shared_matrices or ():
                device.release_matrix(m)
    for a, b in zip(*outs):
        assert a.tobytes() == b.tobytes()

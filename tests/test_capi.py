"""The C-ABI library: it loads, exports every entry point the header declares, and rejects bad arguments before
touching the GPU (no kernel runs here)."""

import ctypes
import os
import re

import pytest

from belt_b200 import _lib, build

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "belt_b200.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(belt_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_lib.lib_path()):
        try:
            build.build()
        except RuntimeError as e:
            pytest.skip(f"cannot build the CUDA library here: {e}")
    return _lib.load()


def test_header_symbols_exported(lib):
    names = declared_functions()
    assert "belt_latent_decode" in names and len(names) >= 8
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.SIGNATURES or n == "belt_last_error", n


def test_abi_version(lib):
    assert lib.belt_abi_version() == 202


def _decode_args(**over):
    a = dict(q_bd=16, num_reqs=1, kq=768, cache=16, num_blocks=4, page=16, row_width=1024, stride_block=16384,
             stride_tok=1024, block_table=16, bt_stride=8, seq_lens=16, work=16, cta_seg=16, num_ctas=148, part=16,
             part_ss=24 * 513, part_sh=513, sm_scale=0.0625, lk_pad=512, lv=512,
             rope_groups=_lib.int_array([0, 64, 128, 64, 256, 64, 384, 64]), rope_blocks=16, n_rope_blocks=4,
             cos_sin=16, max_pos=4096, err=0, stream=0)
    a.update(over)
    return list(a.values())


@pytest.mark.parametrize("bad,msg", [
    (dict(page=24), "page size"),
    (dict(kq=700), "kq"),
    (dict(lv=1000), "lv"),
    (dict(lk_pad=515), "lk_pad"),
    (dict(stride_tok=1020), "16-byte"),
    (dict(n_rope_blocks=3), "rope blocks"),
    (dict(rope_groups=_lib.int_array([0, 64, 128, 64, 256, 64, 480, 64])), "rope group"),
    (dict(q_bd=8), "16-byte"),
])
def test_decode_rejects_bad_arguments(lib, bad, msg):
    rc = lib.belt_latent_decode(*_decode_args(**bad))
    assert rc == -1
    assert msg in lib.belt_last_error().decode()


def test_schedule_rejects_small_capacity(lib):
    rc = lib.belt_decode_schedule(16, 10, 148, 1, 16, 100, 16, 16, 0, 0)
    assert rc == -1 and b"capacity" in lib.belt_last_error()


def test_python_layer_raises_value_error(lib):
    with pytest.raises(ValueError):
        _lib.call("belt_latent_decode", *_decode_args(page=24))


def test_new_entries_reject_bad_arguments(lib):
    """The prefill and model-side entries refuse bad arguments before touching the device."""
    import ctypes
    segs = _lib.int_array([0, 128, 0, 0] * 4)
    # decompress: positions past the request, an unsupported page size
    assert lib.belt_latent_decompress(16, 10, 16, 1024, 16384, 1024, 16, 100, 90, 20, 16, 512, segs, 16, 512, 512,
                                      16, 4096, 16, 16, 1024, 256, 0, 0) == -1
    assert b"outside" in lib.belt_last_error()
    assert lib.belt_latent_decompress(16, 10, 24, 1024, 16384, 1024, 16, 100, 0, 20, 16, 512, segs, 16, 512, 512,
                                      16, 4096, 16, 16, 1024, 256, 0, 0) == -1
    assert b"page size" in lib.belt_last_error()
    # prefill attention: misaligned query, bad strides
    assert lib.belt_prefill_attention(8, 10, 6144, 256, 16, 16, 10, 1024, 256, 0, 0, 1, ctypes.c_float(0.0625), 16,
                                      6144, 256, None, 24, 0, 0) == -1
    assert b"aligned" in lib.belt_last_error()
    # q-norm / RoPE: a rotary width that is not a multiple of 16
    assert lib.belt_q_norm_rope(16, 4, 12288, 512, 16, ctypes.c_float(1e-6), 16, 4096, 24, 16, 1, 16, 6144, 256,
                                0) == -1
    assert b"rot" in lib.belt_last_error()
    # gate: misaligned output
    assert lib.belt_gate_mul(16, 6144, 256, 16, 12288, 512, 4, 8, 6144, 256, 0) == -1
    assert b"aligned" in lib.belt_last_error()

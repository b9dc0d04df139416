"""CPU-side checks of the C ABI: the library builds and loads, exports exactly
what include/gae.h declares, and rejects bad arguments before touching a GPU."""
import ctypes as C
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            txt = open(os.path.join(ROOT, "include", fn)).read()
            names |= set(re.findall(r"GAE_API\s+[\w\s\*]*?\b(gae_\w+)\s*\(", txt))
    return names


def test_library_exports_every_declared_symbol(gae):
    lib = gae.lib()
    names = declared_symbols()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", gae.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (\w+)", out))
    assert names <= exported
    # Nothing but the declared C ABI is exported.
    assert {e for e in exported if not e.startswith("_")} <= names


def test_status_strings(gae):
    L = gae.lib()
    assert L.gae_status_string(0) == b"GAE_OK"
    assert L.gae_status_string(6) == b"GAE_ERR_TIMEOUT"
    assert gae.version().count(".") == 2


def test_attn_rejects_null_args(gae):
    L = gae.lib()
    assert L.gae_attn_fwd(None, None) == 1
    buf = C.create_string_buffer(256)
    assert L.gae_last_error(buf, 256) == 1
    assert b"NULL" in buf.value


def test_attn_rejects_bad_shape(gae):
    a = gae.AttnArgs()
    a.batch, a.heads, a.seq_q, a.seq_kv, a.head_dim = 0, 1, 16, 16, 128
    assert gae.lib().gae_attn_fwd(C.byref(a), None) == 1


def test_attn_rejects_misaligned_stride(gae):
    a = gae.AttnArgs()
    a.q = a.k = a.v = a.o = 1 << 20
    a.batch, a.heads, a.seq_q, a.seq_kv, a.head_dim = 1, 1, 16, 16, 128
    for s in (a.q_stride, a.k_stride, a.v_stride, a.o_stride):
        s[:] = (16 * 130, 16 * 130, 130)  # 130 elements: not a multiple of 16 bytes
    a.dtype = gae.DTYPE_BF16
    a.scale = 0.1
    assert gae.lib().gae_attn_fwd(C.byref(a), None) == 1


def test_attn_rejects_unsupported_head_dim(gae):
    a = gae.AttnArgs()
    a.q = a.k = a.v = a.o = 1 << 20
    a.batch, a.heads, a.seq_q, a.seq_kv, a.head_dim = 1, 1, 16, 16, 80
    for s in (a.q_stride, a.k_stride, a.v_stride, a.o_stride):
        s[:] = (16 * 80, 16 * 80, 80)
    a.dtype = gae.DTYPE_BF16
    a.scale = 0.1
    assert gae.lib().gae_attn_fwd(C.byref(a), None) == 2


def test_empty_host_call_is_ok(gae):
    # seq_len 0: the crate returns an empty Vec; nothing touches the GPU.
    assert gae.lib().gae_waller_operator_f32_host(None, None, None, 0, 64, 1.0, 1, None) == 0


def test_scalar_helpers_match_reference_kats(gae):
    # tests/validation.rs:6-62 against the package's host helpers
    w = gae.WelfordState()
    for x in [2.0, 4.0, 4.0, 4.0, 5.0, 5.0, 7.0, 9.0]:
        w.update(x)
    assert abs(w.mean - 5.0) <= 1e-5 and abs(w.variance() - 4.0) <= 1e-5
    a, b = gae.WelfordState(), gae.WelfordState()
    for x in [1.0, 2.0, 3.0, 4.0]:
        a.update(x)
    for x in [5.0, 6.0, 7.0, 8.0]:
        b.update(x)
    m = gae.WelfordState.merge(a, b)
    assert abs(m.mean - 4.5) <= 1e-5 and abs(m.variance() - 5.25) <= 1e-5
    s = gae.OnlineSoftmax()
    for x in [1.0, 2.0, 3.0, 4.0, 5.0]:
        s.update(x)
    assert abs(s.probability(5.0) - 0.6364086) <= 1e-5
    assert abs(gae.gelu(1.0) - 0.8413) <= 1e-3 and abs(gae.gelu(-1.0) + 0.1587) <= 1e-3
    cfg = gae.GAEConfig.gpt2_small()
    assert (cfg.hidden_dim, cfg.num_heads, cfg.head_dim) == (768, 12, 64)
    llama = gae.GAEConfig.llama_7b()
    assert (llama.hidden_dim, llama.num_heads, llama.head_dim) == (4096, 32, 128)
    with pytest.raises(gae.GAEError):
        gae.GAEConfig.new(100, 3, 400, 16)


def test_symphony_workspace_and_rejections(gae):
    L = gae.lib()
    assert L.gae_symphony_workspace_bytes(1000, 64) == 4 * ((1000 * 64 * 2 + 255) // 256 * 256)
    assert L.gae_symphony_workspace_bytes(0, 64) == 0
    tf = gae.TuningFork.reference_defaults(64)
    assert L.gae_symphony_fwd(None, None, None, None, None, None, None, 16, 64, C.byref(tf),
                              None, None, 0, None) == 1
    p = 1 << 20
    assert L.gae_symphony_fwd(p, p, p, p, p, p, p, 16, 96, C.byref(tf), p, p, 1 << 30, None) == 2
    tf.attn_temperature = 0.0
    assert L.gae_symphony_fwd(p, p, p, p, p, p, p, 16, 64, C.byref(tf), p, p, 1 << 30, None) == 1
    tf.attn_temperature = 1.0
    assert L.gae_symphony_fwd(p, p, p, p, p, p, p, 16, 64, C.byref(tf), p, p, 16, None) == 1


def test_attn_bwd_workspace_and_rejections(gae):
    L = gae.lib()
    assert L.gae_attn_bwd_workspace_bytes(2, 3, 100, 64) == (2 * 3 * 100 * 64 * 4 + 255) // 256 * 256 + \
        (2 * 3 * 100 * 4 + 255) // 256 * 256
    assert L.gae_attn_bwd(None, None) == 1
    a = gae.AttnBwdArgs()
    a.batch, a.heads, a.seq_q, a.seq_kv, a.head_dim = 1, 1, 128, 256, 128
    a.causal = 1
    assert L.gae_attn_bwd(C.byref(a), None) == 2  # causal with seq_q != seq_kv
    a.causal, a.head_dim = 0, 96
    assert L.gae_attn_bwd(C.byref(a), None) == 2
    a.head_dim, a.dtype = 128, 1  # bf16
    assert L.gae_attn_bwd(C.byref(a), None) == 1  # NULL pointers


_STRUCTS = [("gae_attn_args", "AttnArgs"), ("gae_attn_bwd_args", "AttnBwdArgs"),
            ("gae_attn_int8_args", "AttnInt8Args"), ("gae_layer_args", "LayerArgs"),
            ("gae_layer_weights", "LayerWeights"), ("gae_tuning_fork", "TuningFork")]


def test_ctypes_mirrors_match_the_header(gae, tmp_path):
    """Every ctypes mirror in the package has the C struct's size and field
    offsets, as the C compiler lays out include/gae.h."""
    lines = ['#include <stddef.h>', '#include <stdio.h>', '#include "gae.h"', "int main(void) {"]
    for cname, pyname in _STRUCTS:
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in getattr(gae, pyname)._fields_:
            lines.append(f'printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = {}
    for line in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.splitlines():
        cname, key, val = line.split()
        got[(cname, key)] = int(val)
    for cname, pyname in _STRUCTS:
        cls = getattr(gae, pyname)
        assert C.sizeof(cls) == got[(cname, "size")], cname
        for field, _ in cls._fields_:
            assert getattr(cls, field).offset == got[(cname, field)], (cname, field)

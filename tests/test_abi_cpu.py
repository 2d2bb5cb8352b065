"""The C-ABI library: loads without a GPU, exports every symbol of include/spx.h, its
struct layouts match the Python mirror, and host-side validation rejects bad calls
before any launch."""
import ctypes as C
import json
import os
import re
import subprocess
import tempfile

import pytest

from conftest import REPO
from unsloth_spectral import _native as N

HEADER = os.path.join(REPO, "include", "spx.h")


def _declared():
    src = open(HEADER).read()
    return re.findall(r"SPX_API\s+[\w\s\*]+?\b(spx_\w+)\s*\(", src)


def test_library_loads_and_exports_every_declared_symbol():
    lib = N.load()
    names = _declared()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), n
        assert n in N.EXPORTS, f"{n} declared in spx.h but not bound in _native"
    assert lib.spx_abi_version() == N.ABI_VERSION


STRUCTS = {
    "spx_decode_args": N.DecodeArgs,
    "spx_prefill_args": N.PrefillArgs,
    "spx_rsvd_args": N.RsvdArgs,
    "spx_quant_args": N.QuantArgs,
    "spx_reconstruct_args": N.ReconstructArgs,
    "spx_block_score_args": N.BlockScoreArgs,
    "spx_block_value_args": N.BlockValueArgs,
}


def test_struct_layouts_match_header():
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', 'int main(void){', 'printf("{");']
    first = True
    for cname, py in STRUCTS.items():
        for fname, _ in py._fields_:
            sep = "" if first else ","
            first = False
            lines.append(f'printf("{sep}\\"{cname}.{fname}\\":%zu", offsetof({cname}, {fname}));')
        lines.append(f'printf(",\\"{cname}.__size\\":%zu", sizeof({cname}));')
    lines += ['printf("}");', 'return 0;}']
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "probe.c")
        exe = os.path.join(d, "probe")
        open(c, "w").write("\n".join(lines))
        subprocess.run(["gcc", "-std=c11", c, "-o", exe], check=True)
        got = json.loads(subprocess.run([exe], capture_output=True, text=True, check=True).stdout)
    for cname, py in STRUCTS.items():
        for fname, _ in py._fields_:
            assert got[f"{cname}.{fname}"] == getattr(py, fname).offset, (cname, fname)
        assert got[f"{cname}.__size"] == C.sizeof(py), cname


def test_status_strings():
    lib = N.load()
    assert lib.spx_status_string(0) == b"ok"
    assert b"Empty cache" in lib.spx_status_string(N.SPX_ERR_EMPTY)


def _decode_args(**kw):
    a = N.DecodeArgs(num_layers=1, batch=1, num_q_heads=32, num_kv_heads=8, head_dim=128, block_size=512,
                     num_blocks=0, block_capacity=4, rank_k=16, rank_v=16, hot_len=0, hot_capacity=64,
                     dtype=N.SPX_F16, rope_mode=N.SPX_ROPE_ABSOLUTE, rope_tied=1, rope_len=4096,
                     query_position=100, scale=0.088, q=16, out=16, cos_table=16, sin_table=16)
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_decode_host_validation_without_gpu():
    lib = N.load()
    # empty cache is reported before anything touches the device
    assert lib.spx_decode_attn(_decode_args(), None) == N.SPX_ERR_EMPTY
    # GQA mismatch
    assert lib.spx_decode_attn(_decode_args(num_q_heads=30, hot_len=4), None) == 2
    # unsupported head_dim
    assert lib.spx_decode_attn(_decode_args(head_dim=100, hot_len=4), None) == 2
    # cold tier pointers missing
    assert lib.spx_decode_attn(_decode_args(num_blocks=2), None) == 1
    # misaligned codes
    a = _decode_args(num_blocks=2, codes_k=17, codes_v=32, scale_k=32, scale_v=32, basis_k=32, basis_v=32,
                     block_pos=32)
    assert lib.spx_decode_attn(a, None) == 4
    # workspace too small
    a = _decode_args(num_blocks=2, codes_k=32, codes_v=32, scale_k=32, scale_v=32, basis_k=32, basis_v=32,
                     block_pos=32, workspace=256, workspace_bytes=8)
    assert lib.spx_decode_attn(a, None) == 5
    # header + partial records [units][blocks][heads][D + 4] + packed RoPE words [blocks][T][64]
    assert lib.spx_decode_workspace_size(a) == 256 + 1 * 1 * 8 * 2 * 4 * (128 + 4) * 4 + 2 * 512 * 256
    assert b"workspace" in lib.spx_last_error()


def test_rsvd_and_quant_host_validation_without_gpu():
    lib = N.load()
    a = N.RsvdArgs(num_mats=4, m=512, n=128, k=16, r=24, n_iter=2, in_dtype=N.SPX_F16)
    assert lib.spx_rsvd_compress(a, None) == 1          # M / omega missing
    a.M, a.omega = 256, 256
    assert lib.spx_rsvd_compress(a, None) == 5          # no workspace
    assert lib.spx_rsvd_workspace_size(a) > 0
    a.r = 200
    assert lib.spx_rsvd_compress(a, None) == 2          # r too large
    q = N.QuantArgs(num_groups=2, group_elems=0)
    assert lib.spx_quantize_int8(q, None) == 1


def test_rmsnorm_host_validation_without_gpu():
    """spx_rmsnorm rejects bad arguments on the host, before any launch."""
    lib = N.load()
    assert lib.spx_rmsnorm(None, None, 256, 256, None, 4, 4096, 1e-5, N.SPX_BF16, None) == 1       # x missing
    assert lib.spx_rmsnorm(256, 256, 256, 256, None, 4, 4096, 1e-5, N.SPX_BF16, None) == 1        # residual w/o out
    assert lib.spx_rmsnorm(256, None, 256, 256, None, 4, 4100, 1e-5, N.SPX_BF16, None) == 2       # dim % 8
    assert lib.spx_rmsnorm(256, None, 256, 256, None, 4, 16384, 1e-5, N.SPX_BF16, None) == 2      # dim too large
    assert lib.spx_rmsnorm(256, None, 256, 256, None, 4, 4096, 1e-5, N.SPX_F32, None) == 3        # dtype
    assert lib.spx_rmsnorm(264, None, 256, 256, None, 4, 4096, 1e-5, N.SPX_BF16, None) == 4       # alignment
    assert lib.spx_rmsnorm(256, None, 256, 256, None, 0, 4096, 1e-5, N.SPX_BF16, None) == 0       # no rows


def test_rope_rows_host_validation_without_gpu():
    lib = N.load()
    assert lib.spx_rope_rows(None, 1024, 256, 256, 100, None, 0, 5, 256, 2, 8, 128, N.SPX_BF16, None) == 1
    assert lib.spx_rope_rows(256, 1024, 256, 256, 100, None, 0, 5, 256, 2, 8, 127, N.SPX_BF16, None) == 2
    assert lib.spx_rope_rows(256, 512, 256, 256, 100, None, 0, 5, 256, 2, 8, 128, N.SPX_BF16, None) == 2
    assert lib.spx_rope_rows(256, 1024, 256, 256, 100, None, 0, 5, 256, 2, 8, 128, 9, None) == 3
    assert lib.spx_rope_rows(256, 1024, 256, 256, 100, None, 0, 5, 256, 0, 8, 128, N.SPX_BF16, None) == 0


def test_hot_append_host_validation_without_gpu():
    lib = N.load()
    assert lib.spx_hot_append(None, 256, 0, 0, 0, 0, 256, 256, 256, 256, 256, 1, 1, 8, 4, N.SPX_BF16, None) == 1
    assert lib.spx_hot_append(256, 256, 0, 0, 0, 0, 256, 256, 256, 256, 256, 0, 1, 8, 4, N.SPX_BF16, None) == 2
    assert lib.spx_hot_append(256, 256, -1, 0, 0, 0, 256, 256, 256, 256, 256, 1, 1, 8, 4, N.SPX_BF16, None) == 2
    assert lib.spx_hot_append(256, 256, 0, 0, 0, 0, 256, 256, 256, 256, 256, 1, 1, 8, 4, 7, None) == 3


def test_kernels_module_routes_to_library():
    import unsloth_spectral.kernels as K
    assert K.TRITON_AVAILABLE is True
    assert K.TRITON_VERSION.startswith("spx")
    cfg = K.TritonSpectralConfig(enable_logging=False)
    assert cfg.BLOCK_T == 64
    with pytest.raises(AssertionError):
        K.TritonSpectralConfig(BLOCK_T=8)


def test_ops_refuse_cpu_tensors():
    import torch
    from unsloth_spectral import batched_randomized_svd
    with pytest.raises(N.SpxUnavailable):
        batched_randomized_svd(torch.randn(2, 64, 32), 4, oversampling=4)

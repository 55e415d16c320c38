"""The C-ABI library loads and exports every entry point declared in
include/*.h, and the Python binding covers exactly that set (CPU only: no
compute call is made)."""

import ctypes
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _declared() -> set[str]:
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(glm53_\w+)\s*\(", text))
    return names


def test_library_builds_and_exports_every_declared_symbol():
    from glm53_flash_mlx_b200 import _native as N
    from glm53_flash_mlx_b200.build import build

    lib_path = build()
    lib = ctypes.CDLL(str(lib_path))
    declared = _declared()
    assert declared, "no entry points found in include/*.h"
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing
    assert set(N.SIGNATURES) == declared
    loaded = N.load_library()
    assert loaded.glm53_kernel_abi().decode().startswith("glm53-b200-sm100a")
    assert loaded.glm53_last_error() is not None


def test_workspace_queries_are_pure_host_functions():
    from glm53_flash_mlx_b200 import _native as N

    lib = N.load_library()
    assert lib.glm53_packed_decode_workspace_bytes(8, 4096, 1536, 1536) >= (8 * 1536 + 1536) * 2 + 9 * 4096 * 4
    assert lib.glm53_router_workspace_bytes(1, 288) >= 288 * 4
    ws = lib.glm53_grouped_moe_workspace_bytes(2048, 8, 288, 4096, 1536, 1536)
    assert ws >= 16384 * (4096 + 1536) * 2


def test_router_workspace_covers_each_batch_path():
    """glm53_router_workspace_bytes(T, E): logits, sigmoids and keys (T x E each)
    for every T; from 9 to 64 tokens also the FP64 tensor-core tiles' partials
    (up to 8 K ranges x T x E doubles); above 32 the BF16 weight planes
    (3 x E x 8192) of the tcgen05 router as well."""
    from glm53_flash_mlx_b200 import _native as N

    lib = N.load_library()
    E = 288
    for T in (1, 2, 8):
        assert lib.glm53_router_workspace_bytes(T, E) >= 3 * T * E * 4
    for T in (9, 16, 32, 64):
        assert lib.glm53_router_workspace_bytes(T, E) >= 3 * T * E * 4 + 8 * T * E * 8
    for T in (33, 64, 300, 2048):
        assert lib.glm53_router_workspace_bytes(T, E) >= 3 * T * E * 4 + 3 * E * 8192 * 2
    sizes = [lib.glm53_router_workspace_bytes(T, E) for T in range(1, 80)]
    assert sizes == sorted(sizes)  # a workspace sized for T serves every smaller batch


def test_operators_fail_closed_without_cuda():
    import pytest
    import torch

    import glm53_flash_mlx_b200 as G

    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    x = torch.zeros((1, 256), dtype=torch.bfloat16)
    w = torch.zeros((128, 256), dtype=torch.uint8)
    s = torch.ones((1, 2), dtype=torch.float32)
    with pytest.raises(RuntimeError, match="CUDA"):
        G.block_fp8_linear(x, w, s)
    with pytest.raises(RuntimeError):
        G.router_topk(x, torch.zeros((8, 256)), torch.zeros(8), top_k=2)


def test_oracle_library_is_separate_from_product():
    """The product package never imports the oracle."""
    for path in (ROOT / "glm53_flash_mlx_b200").rglob("*.py"):
        text = path.read_text()
        assert "import oracle" not in text and "from oracle" not in text, path


def test_decode_step_descriptor_layout_matches_header(tmp_path):
    """The ctypes mirror of glm53_decode_step_desc has the C struct's size and
    field offsets (gcc compiles the header and prints offsetof for each)."""
    import shutil
    import subprocess

    import pytest

    from glm53_flash_mlx_b200 import _native as N

    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    fields = [f for f, _ in N.DecodeStepDesc._fields_]
    src = tmp_path / "desc.c"
    body = "".join(f'  printf("{f} %zu\\n", offsetof(glm53_decode_step_desc, {f}));\n' for f in fields)
    src.write_text("#include <stddef.h>\n#include <stdio.h>\n#include \"glm53_b200.h\"\nint main(void) {\n"
                   f'  printf("sizeof %zu\\n", sizeof(glm53_decode_step_desc));\n{body}  return 0;\n}}\n')
    exe = tmp_path / "desc"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    got = dict(line.split() for line in subprocess.run([str(exe)], check=True, capture_output=True,
                                                        text=True).stdout.splitlines())
    assert int(got["sizeof"]) == ctypes.sizeof(N.DecodeStepDesc)
    for f in fields:
        assert int(got[f]) == getattr(N.DecodeStepDesc, f).offset, f


def test_new_entry_points_fail_closed_before_touching_cuda():
    """Argument checks of the step, graph-step and batched shared-expert entry
    points reject bad calls with GLM53_ERR_INVALID and a message, before any
    CUDA call (so this runs without a GPU)."""
    from glm53_flash_mlx_b200 import _native as N

    lib = N.load_library()
    assert lib.glm53_graph_step(None, None, None, 0, None, None, 0, None) == N.GLM53_ERR_INVALID
    assert b"glm53_graph_step" in lib.glm53_last_error()
    assert lib.glm53_decode_step_host(None, None, None, None) == N.GLM53_ERR_INVALID
    bad = N.DecodeStepDesc(H=4096, E=288, I=1536, top_k=7)  # no buffers, top_k != 8
    assert lib.glm53_decode_step_host(ctypes.pointer(bad), None, None, None) == N.GLM53_ERR_INVALID
    assert b"glm53_decode_step_host" in lib.glm53_last_error()
    # batched shared-expert entry: missing shared weights / workspace
    assert lib.glm53_batched_decode_moe_shared(None, 2, 4096, None, None, 8, None, None, None, None, 288, 1536,
                                               None, None, None, None, None, None, 10.0, None, None, 0, None, 0,
                                               None) == N.GLM53_ERR_INVALID
    assert b"glm53_batched_decode_moe_shared" in lib.glm53_last_error()
    need = lib.glm53_batched_decode_shared_workspace_bytes(16, 8, 288, 4096, 1536)
    assert need > lib.glm53_batched_decode_workspace_bytes(16, 8, 288, 4096, 1536)

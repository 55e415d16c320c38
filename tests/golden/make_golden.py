"""Regenerate the golden fixtures in this directory.

reference_kats.json -- known answers taken from the reference tree (read as
text/JSON; the reference's MLX code cannot run here):
  * sigmoid sweep: bench-results/m3ultra512-native-routed-sigmoid-formula-
    sweep-20260907.json (domain hash, element count, reference BF16 sigmoid
    hash, the standard-formula hash and its one differing element);
  * E4M3 table: native_execution/native_indexer_plan.metal:18-34 (kNativeE4M3);
  * tile descriptors: tests/test_fp8_metal.py:216-238;
  * packed bank shapes: tests/test_fp8_metal.py:121-124;
  * score recompute: tests/test_grouped_divergence.py:181-199;
  * crossover constants: glm53_flash_mlx/abi.py:5-6.
oracle_small.npz -- outputs of the CPU oracle on small seeded cases, so that a
change of the oracle's arithmetic is visible in review.

Run from the repository root:  python tests/golden/make_golden.py [REFERENCE_ROOT]
"""

from __future__ import annotations

import ast
import json
import os
import re
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))


def reference_kats(ref: Path) -> dict:
    kats: dict = {}
    art = json.loads((ref / "bench-results/m3ultra512-native-routed-sigmoid-formula-sweep-20260907.json").read_text())
    std = art["results"]["standard_bf16"]
    kats["sigmoid_sweep"] = {
        "source": "bench-results/m3ultra512-native-routed-sigmoid-formula-sweep-20260907.json",
        "domain_elements": art["domain"]["elements"],
        "domain_bits_sha256": art["domain"]["bits_sha256"],
        "reference_sigmoid_sha256": art["reference"]["sigmoid_hash"],
        "standard_bf16_sha256": std["actual_hash"],
        "standard_bf16_first_difference": std["first_difference"],
        "standard_bf16_different_elements": std["different_elements"],
    }
    metal = (ref / "native_execution/native_indexer_plan.metal").read_text()
    body = re.search(r"kNativeE4M3\[256\]\s*=\s*\{(.*?)\};", metal, re.S).group(1)
    table = [float(v.strip().rstrip("f")) for v in body.split(",") if v.strip()]
    assert len(table) == 256
    kats["e4m3_table"] = {"source": "native_execution/native_indexer_plan.metal:18-34", "values": table}
    test_src = (ref / "tests/test_fp8_metal.py").read_text()
    m = re.search(r"assert list\(zip\(experts\[valid\].*?\) == (\[.*?\])\n", test_src, re.S)
    kats["tile_descriptors"] = {
        "source": "tests/test_fp8_metal.py:216-238",
        "sorted_experts": {"0": 31, "1": 32, "287": 33},
        "expert_count": 288,
        "tile_rows": 32,
        "valid": [list(t) for t in ast.literal_eval(m.group(1))],
        "unique_experts": 3,
        "zero_route_experts": 285,
    }
    shapes = re.findall(r"assert bank\.(\w+)\.shape == (\([0-9, ]+\))", test_src)
    kats["bank_shapes"] = {
        "source": "tests/test_fp8_metal.py:102-124",
        "hidden_size": 257,
        "intermediate_size": 129,
        "experts": 8,
        "shapes": {name: list(ast.literal_eval(shape)) for name, shape in shapes},
    }
    div_src = (ref / "tests/test_grouped_divergence.py").read_text()
    assert "routed_scaling_factor=2.0" in div_src and "np.array([3.0, 1.0])" in div_src
    raw = 1.0 / (1.0 + np.exp(-np.array([3.0, 1.0])))
    kats["score_recompute"] = {
        "source": "tests/test_grouped_divergence.py:181-199",
        "weight": [[1.0, 0.0], [0.0, 1.0], [1.0, 1.0]],
        "x": [1.0, 2.0],
        "indices": [2, 0],
        "routed_scaling_factor": 2.0,
        "expected_scores": (raw / raw.sum() * 2.0).tolist(),
        "tolerance": 1e-6,
    }
    abi_src = (ref / "glm53_flash_mlx/abi.py").read_text()
    consts = dict(re.findall(r"^(GROUPED_\w+) = (\d+)$", abi_src, re.M))
    kats["abi_constants"] = {"source": "glm53_flash_mlx/abi.py:5-6", **{k: int(v) for k, v in consts.items()}}
    return kats


def small_inputs() -> dict[str, np.ndarray]:
    """Seeded inputs of the small oracle cases (numpy PCG64, reproducible)."""
    import oracle as O

    rng = np.random.default_rng(20260828)
    d: dict[str, np.ndarray] = {}
    d["lin_w"] = rng.integers(0, 247, (129, 257)).astype(np.uint8)
    d["lin_s"] = (rng.uniform(size=(2, 3)) * 0.02).astype(np.float32)
    d["lin_x"] = O.bf16_from_f32(rng.normal(size=(2, 257)).astype(np.float32))
    E, H, I = 8, 257, 129
    d["dec_gu_w"] = rng.integers(0, 247, (E, 2 * I, H)).astype(np.uint8)
    d["dec_gu_s"] = (rng.uniform(size=(E, 4, 3)) * 0.002).astype(np.float32)
    d["dec_d_w"] = rng.integers(0, 247, (E, H, I)).astype(np.uint8)
    d["dec_d_s"] = (rng.uniform(size=(E, 3, 2)) * 0.002).astype(np.float32)
    d["dec_sg_w"] = rng.integers(0, 247, (I, H)).astype(np.uint8)
    d["dec_sg_s"] = (rng.uniform(size=(2, 3)) * 0.002).astype(np.float32)
    d["dec_su_w"] = rng.integers(0, 247, (I, H)).astype(np.uint8)
    d["dec_su_s"] = (rng.uniform(size=(2, 3)) * 0.002).astype(np.float32)
    d["dec_sd_w"] = rng.integers(0, 247, (H, I)).astype(np.uint8)
    d["dec_sd_s"] = (rng.uniform(size=(3, 2)) * 0.002).astype(np.float32)
    d["dec_ids"] = np.array([7, 1, 5, 0, 3, 6, 2, 4], np.uint32)
    d["dec_scores"] = np.array([0.24, 0.18, 0.15, 0.13, 0.11, 0.08, 0.06, 0.05], np.float32)
    d["dec_x"] = O.bf16_from_f32((rng.normal(size=H) * 2).astype(np.float32))
    d["rt_w"] = (rng.normal(size=(32, 256)) * 0.01).astype(np.float32)
    d["rt_b"] = (rng.normal(size=32) * 0.1).astype(np.float32)
    d["rt_x"] = O.bf16_from_f32(rng.normal(size=(4, 256)).astype(np.float32))
    d["rp_ids"] = ((np.arange(96) * 5 + 3) % 8).astype(np.uint32)
    return d


def inputs_digest(d: dict[str, np.ndarray]) -> str:
    import hashlib

    h = hashlib.sha256()
    for k in sorted(d):
        h.update(k.encode())
        h.update(np.ascontiguousarray(d[k]).tobytes())
    return h.hexdigest()


def oracle_small() -> dict[str, np.ndarray]:
    import oracle as O

    d = small_inputs()
    out: dict[str, np.ndarray] = {"inputs_sha256": np.array(inputs_digest(d))}
    out["lin_y2"] = O.block_fp8_linear(d["lin_x"], d["lin_w"], d["lin_s"])
    out["lin_y1"] = O.block_fp8_linear(d["lin_x"][:1], d["lin_w"], d["lin_s"])
    bank = (d["dec_gu_w"], d["dec_gu_s"], d["dec_d_w"], d["dec_d_s"])
    shared = tuple(d["dec_" + n] for n in ("sg_w", "sg_s", "su_w", "su_s", "sd_w", "sd_s"))
    out["dec_y"], out["dec_hidden"] = O.packed_decode_moe(d["dec_x"], d["dec_ids"], d["dec_scores"], bank, shared,
                                                          3.0, return_hidden=True)
    out["rt_idx"], out["rt_scores"], out["rt_logits"], _ = O.router(d["rt_x"], d["rt_w"], d["rt_b"], top_k=8)
    plan = O.route_plan(d["rp_ids"], 8)
    out["rp_order"], out["rp_inverse"], out["rp_offsets"] = plan["order"], plan["inverse"], plan["expert_offsets"]
    return out


def main(argv: list[str]) -> None:
    ref_arg = argv[1] if len(argv) > 1 else os.environ.get("GLM53_REFERENCE_ROOT", "")
    ref = Path(ref_arg) if ref_arg else None
    if ref is not None and ref.exists():
        (HERE / "reference_kats.json").write_text(json.dumps(reference_kats(ref), indent=1) + "\n")
    else:
        print(f"reference tree {ref} absent: reference_kats.json left as committed")
    np.savez_compressed(HERE / "oracle_small.npz", **oracle_small())


if __name__ == "__main__":
    main(sys.argv)

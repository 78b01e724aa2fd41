"""Generate the golden fixtures from the reference's own NumPy oracle.

Run once, in a checkout that has the reference tree (fbaldassarri/mround
0.1.0a6) on ``PYTHONPATH``::

    PYTHONPATH=<mround checkout> python tests/golden/make_golden.py

It imports only the reference's framework-free modules
(``mround/reference/quantize.py``, ``losses.py``, ``optimizer.py``,
``packing.py``, ``mround/planner/sensitivity.py``, ``allocator.py``) and
writes ``tests/golden/golden.npz`` plus ``tests/golden/allocations.json``.
Inputs are float32-representable (weights are bf16 values), so the same
arrays drive the float32 oracle and the CUDA kernels in the tests.
Seeds are fixed; re-running reproduces the files byte for byte.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

from mround.planner import allocator as ref_alloc
from mround.planner import sensitivity as ref_sens
from mround.reference import losses as ref_losses
from mround.reference import optimizer as ref_opt
from mround.reference import packing as ref_pack
from mround.reference import quantize as ref_quant
from mround.reference import scale_search as ref_search
from mround.schemes import QuantScheme, ScaleInit, Symmetry

HERE = Path(__file__).resolve().parent


def bf16_round(x: np.ndarray) -> np.ndarray:
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + (((u >> 16) & 1) + 0x7FFF)) >> 16 << 16
    return (u & 0xFFFFFFFF).astype(np.uint32).view(np.float32)


def sweep_weight(rng: np.random.Generator, rows: int, cols: int) -> np.ndarray:
    """N(0, 0.02) with 0.1 % of entries scaled by 20, rounded to bf16."""
    w = rng.normal(0.0, 0.02, size=(rows, cols))
    hot = rng.random(size=(rows, cols)) < 0.001
    w[hot] *= 20.0
    return bf16_round(w.astype(np.float32))


def quant_cases(out: dict) -> list[str]:
    names = []
    rng = np.random.default_rng(1234)
    for bits in (2, 3, 4, 8):
        for group in (32, 64, 128):
            rows, cols = 12, 256
            w = sweep_weight(rng, rows, cols)
            ng = cols // group
            v = rng.uniform(-0.5, 0.5, size=(rows, cols)).astype(np.float32)
            a = rng.uniform(0.5, 1.0, size=(rows, ng)).astype(np.float32)
            b = rng.uniform(0.5, 1.0, size=(rows, ng)).astype(np.float32)
            gq = rng.normal(0.0, 1e-3, size=(rows, cols)).astype(np.float32)
            scheme = QuantScheme(bits=bits, group_size=group, symmetry=Symmetry.ASYMMETRIC)
            params = ref_quant.QuantParams(
                v.astype(np.float64).reshape(rows, ng, group),
                a.astype(np.float64).reshape(rows, ng, 1),
                b.astype(np.float64).reshape(rows, ng, 1),
            )
            res = ref_quant.fake_quantize(w.astype(np.float64), params, scheme)
            grads = ref_quant.quantize_grad(w.astype(np.float64), params, scheme, gq.astype(np.float64))
            key = f"q_b{bits}_g{group}"
            out[f"{key}_w"] = w
            out[f"{key}_v"] = v
            out[f"{key}_alpha"] = a
            out[f"{key}_beta"] = b
            out[f"{key}_gq"] = gq
            out[f"{key}_qdq"] = res.qdq
            out[f"{key}_codes"] = res.codes.reshape(rows, cols).astype(np.int16)
            out[f"{key}_scale"] = res.scale.reshape(rows, ng)
            out[f"{key}_zp"] = res.zero_point.reshape(rows, ng)
            out[f"{key}_gv"] = grads.v.reshape(rows, cols)
            out[f"{key}_galpha"] = grads.alpha.reshape(rows, ng)
            out[f"{key}_gbeta"] = grads.beta.reshape(rows, ng)
            names.append(key)
    return names


def sym_cases(out: dict) -> list[str]:
    """Symmetric observed-range and searched fake-quant with gradients."""
    names = []
    rng = np.random.default_rng(4321)
    for init in ("observed", "searched"):
        for bits in (2, 3, 4, 8):
            for group in (32, 64, 128):
                rows, cols = 12, 256
                w = sweep_weight(rng, rows, cols)
                ng = cols // group
                v = rng.uniform(-0.5, 0.5, size=(rows, cols)).astype(np.float32)
                lo, hi = (0.5, 1.0) if init == "observed" else (0.5, 1.5)
                a = rng.uniform(lo, hi, size=(rows, ng)).astype(np.float32)
                b = rng.uniform(lo, hi, size=(rows, ng)).astype(np.float32)
                gq = rng.normal(0.0, 1e-3, size=(rows, cols)).astype(np.float32)
                scale_init = ScaleInit.SEARCHED if init == "searched" else ScaleInit.OBSERVED_RANGE
                scheme = QuantScheme(bits=bits, group_size=group, symmetry=Symmetry.SYMMETRIC,
                                     scale_init=scale_init)
                init_scale = None
                if init == "searched":
                    # float32 search result, as the MLX pipeline hands it over
                    init_scale = ref_search.search_scales(w.astype(np.float64), scheme).astype(np.float32)
                params = ref_quant.QuantParams(
                    v.astype(np.float64).reshape(rows, ng, group),
                    a.astype(np.float64).reshape(rows, ng, 1),
                    b.astype(np.float64).reshape(rows, ng, 1),
                )
                base = None if init_scale is None else init_scale.astype(np.float64)
                res = ref_quant.fake_quantize(w.astype(np.float64), params, scheme, init_scale=base)
                grads = ref_quant.quantize_grad(w.astype(np.float64), params, scheme,
                                                gq.astype(np.float64), init_scale=base)
                key = f"s{init[0]}_b{bits}_g{group}"
                out[f"{key}_w"] = w
                out[f"{key}_v"] = v
                out[f"{key}_alpha"] = a
                out[f"{key}_beta"] = b
                out[f"{key}_gq"] = gq
                if init_scale is not None:
                    out[f"{key}_init"] = init_scale.reshape(rows, ng)
                out[f"{key}_qdq"] = res.qdq
                out[f"{key}_codes"] = res.codes.reshape(rows, cols).astype(np.int16)
                out[f"{key}_scale"] = res.scale.reshape(rows, ng)
                out[f"{key}_gv"] = grads.v.reshape(rows, cols)
                out[f"{key}_galpha"] = grads.alpha.reshape(rows, ng)
                out[f"{key}_gbeta"] = grads.beta.reshape(rows, ng)
                names.append(key)
    return names


def search_cases(out: dict) -> list[str]:
    """The scale search, unweighted and importance-weighted, plus edge groups."""
    names = []
    rng = np.random.default_rng(2468)
    for bits in (2, 3, 4, 8):
        for group in (32, 64):
            w = bf16_round(rng.normal(size=(64, 256)).astype(np.float32) * 0.02)
            scheme = QuantScheme(bits=bits, group_size=group)
            key = f"srch_b{bits}_g{group}"
            out[f"{key}_w"] = w
            out[f"{key}_scale"] = ref_search.search_scales(w.astype(np.float64), scheme)
            names.append(key)
    w = bf16_round(rng.normal(size=(32, 64)).astype(np.float32))
    imp = rng.uniform(0.1, 10.0, size=64).astype(np.float32)
    out["srch_imp_w"], out["srch_imp_importance"] = w, imp
    out["srch_imp_scale"] = ref_search.search_scales(
        w.astype(np.float64), QuantScheme(bits=3, group_size=16), importance=imp.astype(np.float64))
    edge = np.zeros((3, 16), dtype=np.float32)
    edge[1, :] = np.linspace(-1.0, 1.0, 16, dtype=np.float32) * 0.01
    edge[2, 3], edge[2, 9] = 0.5, -0.5  # |anchor| tie of opposite signs: first wins
    edge = bf16_round(edge)
    out["srch_edge_w"] = edge
    for bits in (2, 4):
        out[f"srch_edge_b{bits}_scale"] = ref_search.search_scales(
            edge.astype(np.float64), QuantScheme(bits=bits, group_size=16))
    return names


def edge_cases(out: dict) -> None:
    """Single-sign groups, an all-zero group and the clamp-boundary fixture."""
    rows = [
        [-2.0, -1.5, -1.0, -0.5],   # all negative
        [1.0, 1.5, 2.0, 0.25],      # all positive
        [-1.0, 0.0, 1.0, 0.5],      # straddling
        [0.0, 0.0, 0.0, 0.0],       # all zero: scale falls to eps
        [1.0, 0.9, 0.5, -0.3],      # reference boundary fixture
    ]
    w = bf16_round(np.array(rows, dtype=np.float32) * 0.01)
    for bits in (2, 4, 8):
        scheme = QuantScheme(bits=bits, group_size=4, symmetry=Symmetry.ASYMMETRIC)
        params = ref_quant.init_params(w.astype(np.float64), scheme)
        res = ref_quant.fake_quantize(w.astype(np.float64), params, scheme)
        g = np.ones_like(w, dtype=np.float64)
        grads = ref_quant.quantize_grad(w.astype(np.float64), params, scheme, g)
        out[f"edge_b{bits}_w"] = w
        out[f"edge_b{bits}_qdq"] = res.qdq
        out[f"edge_b{bits}_codes"] = res.codes.reshape(w.shape).astype(np.int16)
        out[f"edge_b{bits}_zp"] = res.zero_point.reshape(w.shape[0], 1)
        out[f"edge_b{bits}_gv"] = grads.v.reshape(w.shape)
        out[f"edge_b{bits}_galpha"] = grads.alpha.reshape(w.shape[0], 1)
        out[f"edge_b{bits}_gbeta"] = grads.beta.reshape(w.shape[0], 1)


def optimizer_case(out: dict) -> None:
    """Five signed steps with linear decay and projection on float32 parameters."""
    rng = np.random.default_rng(7)
    rows, cols, group = 8, 128, 64
    ng = cols // group
    v = rng.uniform(-0.5, 0.5, size=(rows, cols)).astype(np.float32)
    a = rng.uniform(0.1, 1.0, size=(rows, ng)).astype(np.float32)
    b = rng.uniform(0.1, 1.0, size=(rows, ng)).astype(np.float32)
    grads = [
        (
            rng.normal(size=(rows, cols)).astype(np.float32),
            rng.normal(size=(rows, ng)).astype(np.float32),
            rng.normal(size=(rows, ng)).astype(np.float32),
        )
        for _ in range(5)
    ]
    # exact zeros must not move a parameter
    grads[0][0][0, :7] = 0.0
    out["opt_v0"], out["opt_a0"], out["opt_b0"] = v, a, b
    for i, (gv, ga, gb) in enumerate(grads):
        out[f"opt_gv{i}"], out[f"opt_ga{i}"], out[f"opt_gb{i}"] = gv, ga, gb
    lr0, iters = 0.05, 5
    scheme = QuantScheme(bits=2, group_size=group, symmetry=Symmetry.ASYMMETRIC)
    opt = ref_opt.SignSGD(ref_opt.LinearDecay(lr0, iters))
    params = ref_quant.QuantParams(
        v.astype(np.float64).reshape(rows, ng, group),
        a.astype(np.float64).reshape(rows, ng, 1),
        b.astype(np.float64).reshape(rows, ng, 1),
    )
    for gv, ga, gb in grads:
        upd = opt.apply(
            {"v": params.v, "alpha": params.alpha, "beta": params.beta},
            {
                "v": gv.astype(np.float64).reshape(rows, ng, group),
                "alpha": ga.astype(np.float64).reshape(rows, ng, 1),
                "beta": gb.astype(np.float64).reshape(rows, ng, 1),
            },
        )
        params = ref_quant.QuantParams(upd["v"], upd["alpha"], upd["beta"])
        ref_quant.project_params(params, scheme)
    out["opt_v5"] = params.v.reshape(rows, cols)
    out["opt_a5"] = params.alpha.reshape(rows, ng)
    out["opt_b5"] = params.beta.reshape(rows, ng)
    out["opt_lr0"] = np.array(lr0)
    out["opt_iters"] = np.array(iters)


def loss_cases(out: dict) -> None:
    rng = np.random.default_rng(11)
    for name, shape in (("small", (2, 16, 64)), ("mid", (4, 64, 96))):
        pred = rng.normal(0.0, 1.0, size=shape).astype(np.float32)
        tgt = (pred + rng.standard_t(3, size=shape) * 0.05).astype(np.float32)
        r = (pred.astype(np.float64) - tgt.astype(np.float64))
        # feed the float32 residual so both sides see identical errors
        r32 = (pred - tgt).astype(np.float64)
        loss_o, grad_o = ref_losses.outlier_suppressed_loss(r32, np.zeros_like(r32))
        loss_m, grad_m = ref_losses.reconstruction_loss(r32, np.zeros_like(r32))
        out[f"loss_{name}_pred"] = pred
        out[f"loss_{name}_tgt"] = tgt
        out[f"loss_{name}_outlier"] = np.array(loss_o)
        out[f"loss_{name}_outlier_grad"] = grad_o
        out[f"loss_{name}_mse"] = np.array(loss_m)
        out[f"loss_{name}_mse_grad"] = grad_m
        del r


def packing_cases(out: dict) -> None:
    rng = np.random.default_rng(5)
    for bits in (2, 3, 4, 5, 6, 7, 8):
        codes = rng.integers(0, 1 << bits, size=(6, 128))
        out[f"pack_b{bits}_codes"] = codes.astype(np.uint8)
        out[f"pack_b{bits}_words"] = ref_pack.pack_codes(codes, bits)


def deltaloss_cases(out: dict) -> None:
    rng = np.random.default_rng(21)
    rows, cols = 32, 192
    w = sweep_weight(rng, rows, cols)
    g = rng.normal(0.0, 1e-2, size=(rows, cols)).astype(np.float32)
    out["dl_w"], out["dl_g"] = w, g
    for bits in (2, 3, 4):
        for group in (32, 64):
            scheme = QuantScheme(bits=bits, group_size=group, symmetry=Symmetry.ASYMMETRIC)
            params = ref_quant.init_params(w.astype(np.float64), scheme)
            q = ref_quant.fake_quantize(w.astype(np.float64), params, scheme).qdq
            out[f"dl_b{bits}_g{group}"] = np.array(ref_sens.delta_loss(w, q, g))


def allocation_cases() -> list[dict]:
    cases = []
    rng = np.random.default_rng(99)
    shapes_pool = [(64, 64), (128, 64), (64, 192), (256, 128), (96, 64)]
    for case in range(6):
        n_layers = 12 + 4 * case
        shapes = {f"model.layers.{i // 7}.l{i % 7}": shapes_pool[rng.integers(len(shapes_pool))]
                  for i in range(n_layers)}
        scores = {}
        for name in shapes:
            base = float(rng.lognormal(0.0, 1.0))
            s2 = base * float(rng.uniform(3.0, 6.0))
            s3 = base * float(rng.uniform(1.2, 2.5))
            scores[name] = {2: s2, 3: s3, 4: base}
            if case == 5 and name.endswith("l0"):
                # exact ties between layers: the argmin must break them identically
                scores[name] = {2: 4.0, 3: 2.0, 4: 1.0}
        scheme = QuantScheme(bits=4, group_size=64, symmetry=Symmetry.ASYMMETRIC)
        average = [2.5, 3.0, 2.25, 3.5, 2.5, 2.75][case]
        budget = ref_sens.mixed_budget_bits(shapes, average, 64)
        options = ref_sens.score_layer_options(scores, shapes, scheme)
        alloc = ref_alloc.allocate_bits(options, budget_bits=budget)
        cases.append({
            "shapes": {k: list(v) for k, v in shapes.items()},
            "scores": {k: {str(b): s for b, s in v.items()} for k, v in scores.items()},
            "average_bits": average,
            "group_size": 64,
            "budget_bits": budget,
            "by_layer": alloc.by_layer,
            "total_cost_bits": alloc.total_cost_bits,
            "predicted_loss": alloc.predicted_loss,
            "average": alloc.average_bits,
        })
    return cases


def main() -> None:
    out: dict[str, np.ndarray] = {}
    names = quant_cases(out)
    out["quant_case_names"] = np.array(names)
    out["sym_case_names"] = np.array(sym_cases(out))
    out["search_case_names"] = np.array(search_cases(out))
    edge_cases(out)
    optimizer_case(out)
    loss_cases(out)
    packing_cases(out)
    deltaloss_cases(out)
    np.savez_compressed(HERE / "golden.npz", **out)
    (HERE / "allocations.json").write_text(json.dumps(allocation_cases(), indent=1) + "\n")
    print(f"wrote {len(out)} arrays")


if __name__ == "__main__":
    main()

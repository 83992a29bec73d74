"""Generate the golden vectors by running the reference implementation.

Run where the reference checkout is available (pure Python, torch CPU):

    python -m tests.golden.make_golden --reference /path/to/int_crush_converter

It rebuilds the seeded inputs of ``cases.py``, runs the reference's own
functions (``converter.rotation``, ``scales``, ``gptq``, ``ldlq``, ``greedy``,
``piso``, ``packing``) on them and writes ``golden.npz`` next to this file.
The reference tree is read only here; tests and the GPU box only need the
committed ``golden.npz``.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--out", default=os.path.join(HERE, "golden.npz"))
    args = ap.parse_args()
    sys.path.insert(0, args.reference)

    import torch
    torch.manual_seed(0)
    from converter import rotation, scales, packing, gptq, ldlq, greedy, piso, rounding

    from tests.golden import cases as C
    from tests.golden import inputs as gi

    out: dict[str, np.ndarray] = {}
    T = torch.from_numpy

    def put(prefix, **kw):
        for k, v in kw.items():
            if isinstance(v, torch.Tensor):
                v = v.detach().cpu().numpy()
            if v is None:
                continue
            out[f"{prefix}/{k}"] = np.asarray(v)

    for n in (16, 64, 256):
        put(f"hadamard_{n}", H=rotation.make_hadamard_regular(n, dtype=torch.float32))
    kat = np.array([0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 0.49999997, -0.49999997, 0.0, -0.0,
                    1e-8, -1e-8, 7.5, -8.5, 3.4999998, -3.4999998, 1e20, -1e20], np.float32)
    put("kat_rhaz", x=kat, y=rounding._round_half_away_from_zero(T(kat)))

    for name, (a, b, n) in C.LINSPACE_CASES.items():
        put(name, v=torch.linspace(a, b, n, dtype=torch.float32))

    for name, c in C.ROT_CASES.items():
        W = gi.weight_outlier_cols(c["seed"], c["M"], c["N"])
        put(name, Wrot=rotation.rotate_weights(T(W), c["rot"]), chk=gi.checksum(W))
    for name, c in C.ROTH_CASES.items():
        H = gi.hessian_lognormal(c["seed"], c["N"], 256)
        if c["nblk"]:
            H = np.stack([H] * c["nblk"]) * np.arange(1, c["nblk"] + 1, dtype=np.float32)[:, None, None]
        put(name, Hrot=rotation.rotate_hessian(T(H), c["rot"]), chk=gi.checksum(H))

    for name, c in C.RTN_CASES.items():
        W = C.rtn_weight(c)
        Ww = rotation.rotate_weights(T(W), c["rot"]) if c["rot"] else T(W)
        gs = c["gs"] or Ww.shape[1]
        if c["bits"] == 4 and not c["asym"]:
            s = scales.calculate_scales(Ww, gs, clipping_ratios=c["ratios"])
            q = scales.quantize_weights(Ww, s, gs)
            zp = None
        elif c["bits"] == 4:
            s, zp = scales.calculate_scales_asymmetric(Ww, gs, clipping_ratios=c["ratios"])
            q = scales.quantize_weights_asymmetric(Ww, s, zp, gs)
        elif not c["asym"]:
            s = scales.calculate_scales_int8(Ww, clipping_ratios=c["ratios"])
            q = scales.quantize_weights_int8(Ww, s)
            zp = None
        else:
            s, zp = scales.calculate_scales_int8_asymmetric(Ww, clipping_ratios=c["ratios"])
            q = scales.quantize_weights_int8_asymmetric(Ww, s, zp)
        put(name, scales=s, zp=zp, codes=q, chk=gi.checksum(W))
        if c["bits"] == 4:
            put(name, packed=packing.pack_int4(q))

    for name, c in C.PACK_CASES.items():
        q = gi.codes(c["seed"], c["M"], c["K"])
        put(name, packed=packing.pack_int4(T(q)))

    for name, c in C.GPTQ_CASES.items():
        W, H = C.gptq_inputs(c)
        Ww = rotation.rotate_weights(T(W), c["rot"]) if c["rot"] else T(W)
        Hr = rotation.rotate_hessian(T(H), c["rot"]) if c["rot"] else T(H)
        r = gptq.gptq_quantize_layer(Ww, Hr, block_size=c["bs"], damping=0.01, int_bits=c["bits"],
                                     asymmetric=c["asym"])
        Qn = r.quantized_W.numpy()
        zp = r.zero_points
        s32 = np.asarray(r.scales.float().numpy(), np.float64)
        E = Ww.double().numpy() - (Qn.astype(np.float64) - (zp.double().numpy() if zp is not None else 0.0)) * s32
        if Hr.dim() == 2:
            proxy = float(np.einsum("ij,ij->", E @ Hr.double().numpy(), E))
        else:
            bs = Hr.shape[1]
            proxy = sum(float(np.einsum("ij,ij->", E[:, i * bs:(i + 1) * bs] @ Hr[i].double().numpy(),
                                        E[:, i * bs:(i + 1) * bs])) for i in range(Hr.shape[0]))
        put(name, codes=r.quantized_W, scales=r.scales, zp=zp, mse=np.float64(r.mse),
            max_err=np.float64(r.max_err), proxy=np.float64(proxy), chk=gi.checksum(W, H))
        if c["N"] <= 64:
            put(name, Hinv=gptq._prepare_hinv(Hr, 0.01, torch.device("cpu")))

    for name, c in C.LDLQ_CASES.items():
        W, H = C.ldlq_inputs(c)
        Ww = rotation.rotate_weights(T(W), c["rot"]) if c["rot"] else T(W)
        Hr = None if H is None else (rotation.rotate_hessian(T(H), c["rot"]) if c["rot"] else T(H))
        r = ldlq.ldlq_quantize_layer(Ww, hessian=Hr, block_size=c["bs"], damping=0.01,
                                     int_bits=c["bits"], iterations=c["iters"], greedy_passes=c["greedy"])
        Wd = Ww.double().numpy()
        Hp = Hr.double().numpy() if Hr is not None else Wd.T @ Wd / Wd.shape[0]
        E = Wd - r.quantized_W.numpy().astype(np.float64) * r.scales.double().numpy()
        proxy = float(np.einsum("ij,ij->", E @ Hp, E))
        put(name, codes=r.quantized_W, scales=r.scales, mse=np.float64(r.mse), proxy=np.float64(proxy),
            chk=gi.checksum(W))

    for name, c in C.GREEDY_CASES.items():
        W, Q, S, H = C.greedy_inputs(c)
        qmin, qmax = (-8, 7) if c["bits"] == 4 else (-128, 127)
        Qo = greedy.greedy_local_search_pytorch(T(W), T(Q).float().contiguous(), T(S), T(H),
                                                c["passes"], qmin, qmax)
        put(name, codes=Qo, chk=gi.checksum(W, Q, S, H))

    for name, c in C.PISO_CASES.items():
        W, hd = C.piso_inputs(c)
        k = c["kind"]
        if k == "int8":
            put(name, scales=piso._compute_piso_scales_pytorch(T(W), T(hd), 128, 16, -128, 127, 127.0))
        elif k == "int4":
            put(name, scales=piso._compute_piso_scales_pytorch(T(W), T(hd), 128, 16, -8, 7, 7.0))
        elif k == "int8_asym":
            s, zp = piso._compute_piso_scales_asymmetric_pytorch(T(W), T(hd), 128, 16, -128, 127, 0.8, 1.2)
            put(name, scales=s, zp=zp)
        else:
            s, zp = piso._compute_piso_scales_asymmetric_pytorch(T(W), T(hd), 128, 16, -8, 7, 0.5, 2.0)
            put(name, scales=s, zp=zp)
        put(name, chk=gi.checksum(W, hd))

    from converter import smoothquant
    from converter import pipeline
    for name, c in C.SMOOTH_CASES.items():
        W, H, s = C.smooth_inputs(c)
        put(name, W_smooth=smoothquant.apply_smoothing_to_weight(T(W), T(s)),
            H_smooth=pipeline._transform_hessian_for_smoothquant(T(H), T(s)), chk=gi.checksum(W, H, s))


    for name, c in C.GPTQ_EXTRA_CASES.items():
        W, H, ps, pz = C.gptq_extra_inputs(c)
        kw = dict(int_bits=c["bits"], asymmetric=c["asym"])
        if ps is not None:
            kw.update(piso_scales=T(ps), piso_zero_points=None if pz is None else T(pz))
        if c["kind"] == "rtn":
            r = gptq.gptq_quantize_layer_rtn(T(W), clipping_ratios=c.get("ratios"), **kw)
        else:
            if isinstance(H, dict):
                Hin = {"format": "dlr", "D": T(H["D"]), "U": T(H["U"])}
            else:
                Hin = T(H)
            method = "cholesky" if c["kind"] == "cholesky" else "hinv"
            r = gptq.gptq_quantize_layer(T(W), Hin, block_size=128, damping=0.01, hessian_method=method, **kw)
        put(name, codes=r.quantized_W, scales=r.scales, zp=r.zero_points, mse=np.float64(r.mse),
            max_err=np.float64(r.max_err), method=np.array(r.method_used), chk=gi.checksum(W))
        if c["kind"] == "dlr":
            from converter import dlr
            put(name, Hinv=dlr.woodbury_inverse(T(H["D"]), T(H["U"]), damping=0.01))

    for name, c in C.ROTACT_CASES.items():
        rng = np.random.default_rng(c["seed"])
        x = rng.standard_normal(c["shape"]).astype(np.float32)
        put(name, y=rotation.rotate_activations(T(x), c["rot"]))

    for name, c in C.SQ_CASES.items():
        W, hd = C.sq_inputs(c)
        if c["nsamp"]:
            put(name, s=smoothquant.compute_smoothing_from_hessian_diag(T(hd), T(W), alpha=c["alpha"],
                                                                       num_calibration_samples=c["nsamp"]))
        else:
            put(name, s=smoothquant.compute_smoothing_factors(T(hd), T(W), alpha=c["alpha"]))


    from converter import permuquant
    for name, c in C.PQ_CASES.items():
        W, act = C.pq_inputs(c)
        Wt = T(W)
        at = None if act is None else T(act)
        mu2 = permuquant.channel_second_moments(Wt)
        if act is None:
            perm = permuquant.find_permutation_weight(Wt, c["group"])
        else:
            perm = permuquant.find_permutation_joint(Wt, at, 0.5, c["group"])
        e0 = permuquant.compute_group_quant_error(Wt, c["group"], c["bits"])
        e1 = permuquant.compute_group_quant_error(Wt[:, perm], c["group"], c["bits"])
        p2, acc = permuquant.find_permutation_with_acceptance(Wt, at, 0.5, c["group"], 0.0, c["bits"])
        put(name, mu2=mu2, perm=perm, err=np.float64(e0), err_perm=np.float64(e1), accepted=np.array(bool(acc)),
            chk=gi.checksum(W))


    from converter import svd
    for name, c in C.SVD_CASES.items():
        W = C.svd_inputs(c)
        torch.manual_seed(0)
        r = svd.decompose_weight(T(W), rank=c["rank"])
        put(name, res_energy=np.float64((r.residual.double() ** 2).sum().item()),
            L1_shape=np.array(r.L1.shape), L2_shape=np.array(r.L2.shape), chk=gi.checksum(W))

    np.savez_compressed(args.out, **out)
    print(f"wrote {len(out)} arrays to {args.out} ({os.path.getsize(args.out)} bytes)")


if __name__ == "__main__":
    main()

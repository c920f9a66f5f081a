"""Generate golden vectors by running the REFERENCE's own CUDA extensions on a B200.

The reference (inEXASCALE/euclid-cuda) has no tests or fixtures of its own, so its
behaviour is pinned here: its six extensions are compiled from the unmodified
sources by oracle/build_ref.py into oracle/_ref/, and this script feeds them
seeded inputs and stores inputs + outputs as small .npz files next to it.  The
CPU oracle is checked against these files (tests/test_oracle_golden.py) and the
engine against both.

Usage (on a B200):  python tests/golden/make_golden.py [--out tests/golden]

Shapes avoid the reference's known hazards: N and M are multiples of 32 for the
tiled kernels (a partial tile reaches a divergent __syncthreads,
euclidean_kernels_tiled.cu:145-148 vs :177,189), tensor-core ops get tile_size=32
and dim % 16 == 0, and N*M stays far below 2^31.
"""
import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.path.join(REPO, "oracle", "_ref")

MIX = ["fp16_fp64", "bf16_fp64", "tf32_fp64", "fp32_fp64", "fp16_fp16", "fp16_fp32", "bf16_bf16", "bf16_fp32",
       "fp32_fp32"]
TILED = ["fp16_fp64", "fp16_fp32", "bf16_fp64", "bf16_fp32", "fp32_fp64", "fp32_fp32"]
TC = ["fp16_fp64", "fp16_fp32", "bf16_fp64", "bf16_fp32"]
UNIFORM = ["fp16", "bf16", "tf32", "fp16_direct", "bf16_direct", "tf32_direct", "fp32_direct", "fp64_direct"]
ADV = ["fp64_fp16", "fp64_bf16", "fp64_tf32", "fp64_fp32_gemm"]


def blobs(rng, n, m, d, noise, offset=0.0, scale=1.0):
    """m centers ~ N(0, scale^2) (+offset); points = random center + N(0, noise^2)."""
    C = rng.normal(0.0, scale, (m, d)) + offset
    lab = rng.integers(0, m, n)
    P = C[lab] + rng.normal(0.0, noise, (n, d))
    return P.astype(np.float32), C.astype(np.float32)


def cases():
    rng = np.random.default_rng(20261201)
    out = []
    # name, P, C : fp32 inputs
    P, C = blobs(rng, 96, 64, 40, 0.05)
    out.append(("blobs_96x64x40", P, C))
    P, C = blobs(rng, 64, 32, 16, 0.5)
    out.append(("blobs_64x32x16", P, C))
    P = rng.normal(size=(128, 48)).astype(np.float32)
    C = rng.normal(size=(64, 48)).astype(np.float32)
    out.append(("gauss_128x64x48", P, C))
    # cancellation stress: large common offset, tiny spread (C3-like)
    P, C = blobs(rng, 64, 32, 32, 0.01, offset=1000.0, scale=0.1)
    out.append(("offset_64x32x32", P, C))
    # ties and exact zeros: duplicated centers, points equal to centers
    C = rng.normal(size=(32, 16)).astype(np.float32)
    C[5] = C[3]
    C[20] = C[3]
    P = np.concatenate([C[:16], rng.normal(size=(16, 16)).astype(np.float32)], 0)
    out.append(("ties_32x32x16", P, C))
    # fp16 overflow of norms/products (values ~300, d=32 -> |p|^2 ~ 2.9e6 > 65504)
    P, C = blobs(rng, 32, 32, 32, 1.0, offset=300.0, scale=1.0)
    out.append(("overflow16_32x32x32", P, C))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=HERE)
    a = ap.parse_args()
    import torch
    sys.path.insert(0, REF)
    import ref_center_kernels as rcen
    import ref_euclidean_advanced as radv
    import ref_euclidean_cuda as rbase
    import ref_euclidean_mix as rmix
    import ref_euclidean_tiled as rtil
    import ref_euclidean_uniform as runi

    dev = torch.device("cuda:0")
    kappas = [5.0, 0.05]
    for name, P, C in cases():
        rec = {"P": P, "C": C, "kappas": np.array(kappas, np.float32)}
        Pt, Ct = torch.from_numpy(P).to(dev), torch.from_numpy(C).to(dev)
        rec["single"] = rbase.pairwise_euclidean_single(Pt, Ct).cpu().numpy()
        rec["double"] = rbase.pairwise_euclidean_double(Pt.double(), Ct.double()).cpu().numpy()
        for ki, kappa in enumerate(kappas):
            for op in MIX:
                D, cnt = getattr(rmix, f"pairwise_euclidean_{op}_with_stats")(Pt, Ct, kappa)
                rec[f"mix_{op}_k{ki}"] = D.cpu().numpy()
                rec[f"mix_{op}_k{ki}_count"] = np.array(cnt, np.int64)
            if P.shape[0] % 32 == 0 and C.shape[0] % 32 == 0:
                for op in TILED:
                    for T in (16, 32):
                        if P.shape[1] > 512:
                            continue
                        D, tot, per = getattr(rtil, f"pairwise_euclidean_tiled_{op}_with_stats")(Pt, Ct, kappa, T)
                        rec[f"tiled_{op}_T{T}_k{ki}"] = D.cpu().numpy()
                        rec[f"tiled_{op}_T{T}_k{ki}_tiles"] = np.array(per, np.int64)
                if P.shape[1] % 16 == 0:
                    for op in TC:
                        D = getattr(rtil, f"pairwise_euclidean_tensorcore_{op}")(Pt, Ct, kappa, 32)
                        torch.cuda.synchronize()
                        rec[f"tc_{op}_k{ki}"] = D.cpu().numpy()
            for op in ADV:
                if op == "fp64_fp16":
                    args = (Pt.half(), Ct.half())
                elif op == "fp64_bf16":
                    args = (Pt.bfloat16(), Ct.bfloat16())
                elif op == "fp64_tf32":
                    args = (Pt, Ct)
                else:
                    args = (Pt.double(), Ct.double())
                D = getattr(radv, f"pairwise_euclidean_{op}")(*args, kappa)
                rec[f"adv_{op}_k{ki}"] = D.cpu().numpy()
        for op in UNIFORM:
            if op.startswith("fp16"):
                args = (Pt.half(), Ct.half())
            elif op.startswith("bf16"):
                args = (Pt.bfloat16(), Ct.bfloat16())
            elif op.startswith("fp64"):
                args = (Pt.double(), Ct.double())
            else:
                args = (Pt, Ct)
            D = getattr(runi, f"pairwise_euclidean_uniform_{op}")(*args)
            if D.dtype == torch.bfloat16:
                rec[f"uni_{op}"] = D.view(torch.int16).cpu().numpy().view(np.uint16)
            else:
                rec[f"uni_{op}"] = D.cpu().numpy()
        # inputs in the low formats, as the reference saw them
        rec["P_bf16"] = Pt.bfloat16().view(torch.int16).cpu().numpy().view(np.uint16)
        rec["C_bf16"] = Ct.bfloat16().view(torch.int16).cpu().numpy().view(np.uint16)
        # caller-side argmin of a reference D, and the center update on those labels
        lab = torch.from_numpy(rec["mix_fp16_fp32_k0"]).to(dev).argmin(1)
        rec["argmin_mix_fp16_fp32_k0"] = lab.cpu().numpy()
        k = C.shape[0]
        rec["centers_fp32"] = rcen.update_centers_fp32(Pt, lab, k).cpu().numpy()
        rec["centers_fp64"] = rcen.update_centers_fp64(Pt.double(), lab, k).cpu().numpy()
        rec["centers_labels"] = lab.cpu().numpy()
        np.savez_compressed(os.path.join(a.out, f"{name}.npz"), **rec)
        print(f"[golden] {name}: {len(rec)} arrays", flush=True)
    # center update with empty clusters and out-of-range labels
    rng = np.random.default_rng(7)
    X = rng.normal(size=(500, 8)).astype(np.float32)
    lab = rng.integers(0, 10, 500)
    lab[lab == 4] = 3           # cluster 4 empty
    lab[:5] = 12                # out of range: ignored
    lab[5:8] = -1
    Xt = torch.from_numpy(X).to(dev)
    lt = torch.from_numpy(lab.astype(np.int64)).to(dev)
    np.savez_compressed(os.path.join(a.out, "centers_empty.npz"), X=X, labels=lab.astype(np.int64),
                        centers_fp32=rcen.update_centers_fp32(Xt, lt, 10).cpu().numpy(),
                        centers_fp64=rcen.update_centers_fp64(Xt.double(), lt, 10).cpu().numpy())
    print("[golden] centers_empty", flush=True)


if __name__ == "__main__":
    main()

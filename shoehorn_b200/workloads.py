"""Synthetic inputs of the benchmark configurations (no network, so seeded
stand-ins with the configurations' shapes and distributions replace model
weights and real imatrices).

  sweep tensor   4096 rows x 14336 BF16: N(0, 0.02) with 0.1% of the
                 elements set to +-8 sigma (+-0.16), per-column log-normal
                 imatrix exp(N(0, 1.5)).
  IQ tensors     [4096 rows x 4096] and [14336 rows x 4096] BF16: Student-t
                 (nu = 5) scaled to std 0.02, per-column imatrix exp(N(0, 1)).

BF16 is the round-to-nearest-even rounding of the f32 draw.  Both bench.py
and the parity tests draw from here, so the tests cover the benchmark data.
"""
import numpy as np

SEED = 20261201
SWEEP_SHAPE = (4096, 14336)
IQ_SHAPES = ((4096, 4096), (14336, 4096))


def to_bf16(w):
    """f32 array -> BF16 bit patterns (uint16), round to nearest even."""
    u = np.ascontiguousarray(w, dtype=np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def sweep_tensor(seed=SEED, n_rows=SWEEP_SHAPE[0], ne0=SWEEP_SHAPE[1]):
    """(bf16 bits [n_rows, ne0], imatrix [ne0]) of the encoder sweep."""
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((n_rows, ne0), dtype=np.float32)
    w *= np.float32(0.02)
    k = int(round(w.size * 0.001))
    idx = rng.choice(w.size, size=k, replace=False)
    w.reshape(-1)[idx] = rng.choice(np.array([-0.16, 0.16], dtype=np.float32), size=k)
    im = np.exp(rng.normal(0.0, 1.5, size=ne0)).astype(np.float32)
    return to_bf16(w), im


def iq_tensors(seed=SEED):
    """[(name, bf16 bits, imatrix)] of the IQ codebook configuration."""
    out = []
    for i, (rows, ne0) in enumerate(IQ_SHAPES):
        rng = np.random.default_rng(seed + 1 + i)
        w = (rng.standard_t(5.0, size=(rows, ne0)) * (0.02 / np.sqrt(5.0 / 3.0))).astype(np.float32)
        im = np.exp(rng.normal(0.0, 1.0, size=ne0)).astype(np.float32)
        out.append((f"{rows}x{ne0}", to_bf16(w), im))
    return out


def main(argv=None):
    """Encode a sample of a benchmark workload on cuda:0 a few times (a small,
    repeatable launch for profilers):

      python -m shoehorn_b200.workloads --type 14 --rows 512 [--dist iq] [--repeat 2]

    --table STEP computes the fused error table (row_errors) of every STEP-th
    row instead of encoding.
    """
    import argparse
    ap = argparse.ArgumentParser(prog="python -m shoehorn_b200.workloads")
    ap.add_argument("--type", type=int, required=True, help="ggml type id")
    ap.add_argument("--rows", type=int, default=512)
    ap.add_argument("--dist", choices=["sweep", "iq"], default="sweep",
                    help="sweep: N(0, 0.02) + outliers, 14336 wide; iq: Student-t, 4096 wide")
    ap.add_argument("--repeat", type=int, default=2)
    ap.add_argument("--table", type=int, default=0, metavar="STEP",
                    help="fused error table of every STEP-th row instead of the encode")
    args = ap.parse_args(argv)
    import torch
    import shoehorn_b200 as sh
    if args.dist == "sweep":
        bits, im = sweep_tensor(n_rows=args.rows)
    else:
        rng = np.random.default_rng(5)
        w = (rng.standard_t(5.0, size=(args.rows, 4096)) * (0.02 / np.sqrt(5.0 / 3.0))).astype(np.float32)
        bits, im = to_bf16(w), np.exp(rng.normal(0.0, 1.0, size=4096)).astype(np.float32)
    with sh.Context(0) as ctx:
        src = torch.from_numpy(bits.view(np.int16)).cuda()
        imt = torch.from_numpy(im).cuda()
        for _ in range(args.repeat):
            if args.table:
                ctx.row_errors([args.type], src, imt, row_step=args.table, sync=True)
            else:
                ctx.encode_rows(args.type, src, imt, sync=True)
    what = f"error table (row step {args.table})" if args.table else "encoded"
    print(f"{what} {args.rows} x {bits.shape[1]} to type {args.type} x{args.repeat}")


if __name__ == "__main__":
    main()

"""GPU pipeline: the reference's end-to-end test (e2e_tests.rs:117-187) through
the shoehorn-gpu CLI, and the whole plan/quantize output checked against the
oracle: the same candidate errors, the same solver picks, the same tensor
bytes."""
import os
import subprocess

import numpy as np
import pytest

from oracle import oracle as O
from tests import solver_ref

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
gguf = pytest.importorskip("gguf")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLI = os.path.join(ROOT, "shoehorn_b200", "shoehorn-gpu")
T = {"F32": 0, "F16": 1, "Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "IQ2_XXS": 16, "IQ2_XS": 17,
     "IQ3_XXS": 18, "IQ4_NL": 20, "IQ3_S": 21, "IQ2_S": 22, "IQ4_XS": 23, "BF16": 30}
NAME = {v: k for k, v in T.items()}


def run(*args):
    r = subprocess.run([CLI, *args], capture_output=True, text=True, timeout=1800)
    assert r.returncode == 0, r.stderr[-2000:]
    return r


def ladder(name, ne0):
    """main.rs:347-380 dispose for a 2-D .weight tensor."""
    if ne0 % 256 == 0:
        c = ["IQ4_XS", "Q4_K", "Q5_K", "Q6_K", "Q8_0"]
        if name not in ("token_embd.weight", "output.weight"):
            c += ["IQ2_XXS", "IQ2_XS", "IQ2_S", "IQ3_XXS", "IQ3_S"]
    else:
        c = ["IQ4_NL", "Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q8_0"]
    c.append("F16")
    return sorted(c, key=lambda t: O.row_bytes(T[t], ne0))  # stable, like sort_by_key


@pytest.fixture(scope="module")
def e2e(tmp_path_factory):
    d = tmp_path_factory.mktemp("e2e")
    src = str(d / "synthetic-bf16.gguf")
    run("synth", "e2e", src)
    return d, src


def test_pipeline_fits_a_synthetic_model_into_a_tight_budget(e2e):
    d, src = e2e
    out = str(d / "synthetic-fit.gguf")
    overhead, room = 64 * 1024 + 576 * 1024, 200 * 1024
    r = run("quantize", "-m", src, "-o", out, "--ctx", "64", "--budget", str(overhead + room), "--reserve", "0",
            "--exact-errors")
    model_budget = room
    ref = gguf.GGUFReader(src)
    fit = gguf.GGUFReader(out)
    total = sum(int(t.n_bytes) for t in fit.tensors)
    assert total <= model_budget
    assert total >= model_budget * 0.85
    assert any(t.tensor_type.name not in ("F16", "F32") for t in fit.tensors)
    assert [t.name for t in fit.tensors] == [t.name for t in ref.tensors]
    assert [list(t.shape) for t in fit.tensors] == [list(t.shape) for t in ref.tensors]
    assert "general.file_type" in fit.fields and "general.quantization_version" in fit.fields
    arch = fit.fields["general.architecture"]
    assert bytes(arch.parts[arch.data[0]]).decode() == "llama"
    for t in fit.tensors:
        vals = gguf.quants.dequantize(np.asarray(t.data), t.tensor_type)
        assert np.all(np.isfinite(vals)), t.name
    assert "timing:" in r.stderr


def oracle_plan(src, budget_weights):
    """Error table, solve and bytes of the e2e fixture by the oracle."""
    rd = gguf.GGUFReader(src)
    fixed_bytes, choices, fixed = 0, [], {}
    for t in rd.tensors:
        dims = [int(x) for x in t.shape]
        ne0, n_rows = dims[0], int(np.prod(dims[1:])) if len(dims) > 1 else 1
        if len(dims) >= 2 and t.name.endswith(".weight") and ne0 % 32 == 0:
            bits = np.asarray(t.data).reshape(-1).view(np.uint16).reshape(n_rows, ne0)
            cands = []
            for ty in ladder(t.name, ne0):
                e = O.row_errors_bf16(T[ty], bits, None, row_step=1)
                err = 0.0
                for v in e:
                    err += float(v)
                cands.append((O.row_bytes(T[ty], ne0) * n_rows, err * (n_rows / n_rows), ty, bits))
            choices.append((t.name, cands))
        else:
            fixed[t.name] = "F32"
            fixed_bytes += 4 * ne0 * n_rows
    sel = solver_ref.solve([[(c[0], c[1]) for c in cs] for _, cs in choices], budget_weights - fixed_bytes)
    return {name: cs[i] for (name, cs), i in zip(choices, sel)}, fixed


def test_plan_and_bytes_match_the_oracle(e2e):
    d, src = e2e
    out = str(d / "fit-oracle.gguf")
    overhead, room = 64 * 1024 + 576 * 1024, 200 * 1024
    run("quantize", "-m", src, "-o", out, "--ctx", "64", "--budget", str(overhead + room), "--reserve", "0",
        "--exact-errors")
    picks, fixed = oracle_plan(src, room)
    fit = gguf.GGUFReader(out)
    for t in fit.tensors:
        if t.name in fixed:
            assert t.tensor_type.name == "F32"
            continue
        nbytes, err, ty, bits = picks[t.name]
        assert t.tensor_type.name == ty, t.name
        want = O.encode_tensor_bf16(T[ty], bits, None)
        assert np.array_equal(np.asarray(t.data).reshape(-1).view(np.uint8), want.reshape(-1)), t.name


def test_sampled_errors_and_imatrix_plan_match_the_oracle(tmp_path):
    """Default 128-row sampling (main.rs:546) with an imatrix, on a model
    whose tensors have more than 128 rows."""
    src, im = str(tmp_path / "tiny.gguf"), str(tmp_path / "tiny.imatrix")
    run("synth", "tiny", src, "--imatrix", im)
    out = str(tmp_path / "tiny-fit.gguf")
    r = run("quantize", "-m", src, "-i", im, "-o", out, "--ctx", "64", "--budget", "1600000", "--reserve", "0")
    rd, fit = gguf.GGUFReader(src), gguf.GGUFReader(out)
    # the legacy imatrix as the pipeline reads it (ncall = 1, positive values)
    import struct
    ims = {}
    with open(im, "rb") as f:
        n = struct.unpack("<i", f.read(4))[0]
        for _ in range(n):
            ln = struct.unpack("<i", f.read(4))[0]
            name = f.read(ln).decode()
            _, nv = struct.unpack("<ii", f.read(8))
            ims[name] = np.frombuffer(f.read(4 * nv), np.float32).copy()
    fitted = {t.name: t for t in fit.tensors}
    for t in rd.tensors:
        dims = [int(x) for x in t.shape]
        if len(dims) < 2:
            continue
        ne0, n_rows = dims[0], int(np.prod(dims[1:]))
        bits = np.asarray(t.data).reshape(-1).view(np.uint16).reshape(n_rows, ne0)
        tim = ims.get(t.name[:-len(".weight")])
        ft = fitted[t.name]
        want = O.encode_tensor_bf16(T[ft.tensor_type.name], bits, tim)
        assert np.array_equal(np.asarray(ft.data).reshape(-1).view(np.uint8), want.reshape(-1)), t.name
    assert "weights:" in r.stdout


def test_uniform_mix_harness(tmp_path):
    src = str(tmp_path / "e2e.gguf")
    run("synth", "e2e", src)
    out = str(tmp_path / "u.gguf")
    run("quantize", "-m", src, "-o", out, "--uniform", "Q4_K,token_embd.weight=Q6_K")
    fit = gguf.GGUFReader(out)
    for t in fit.tensors:
        if len(t.shape) < 2:
            assert t.tensor_type.name == "F32"
        elif t.name == "token_embd.weight":
            assert t.tensor_type.name == "Q6_K"
        else:
            assert t.tensor_type.name == "Q4_K"


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_sharding_gives_identical_output(tmp_path):
    src, im = str(tmp_path / "tiny.gguf"), str(tmp_path / "tiny.imatrix")
    run("synth", "tiny", src, "--imatrix", im)
    outs = []
    for g in (1, 2):
        out = str(tmp_path / f"g{g}.gguf")
        run("quantize", "-m", src, "-i", im, "-o", out, "--ctx", "64", "--budget", "1600000", "--reserve", "0",
            "--exact-errors", "--gpus", str(g))
        outs.append(open(out, "rb").read())
    assert outs[0] == outs[1]


def test_streamed_model_writes_the_same_file(tmp_path):
    """A model whose rows are generated as the pipeline asks for them (how
    the 70B shape runs without holding its weights) plans and writes the
    same GGUF, byte for byte, as the same model held in memory."""
    from shoehorn_b200 import host
    budget = str(64 * 1024 + 576 * 1024 + 400 * 1024)  # KV + compute at ctx 64, then 400 KiB of weights
    files = []
    for streaming in (False, True):
        out = str(tmp_path / f"tiny-{int(streaming)}.gguf")
        recs = host.bench_model("tiny", modes=("sampled", "exact"), budget=budget, reserve="0", ctx=64,
                                out_path=out, streaming=streaming)
        assert [r["streaming"] for r in recs] == [streaming, streaming]
        files.append(open(out, "rb").read())
    assert files[0] == files[1]
    fit = gguf.GGUFReader(str(tmp_path / "tiny-1.gguf"))
    assert any(t.tensor_type.name not in ("F16", "F32") for t in fit.tensors)

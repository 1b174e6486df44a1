"""Shared fixtures.  `gpu`-marked tests need a B200; the rest run on CPU."""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def native():
    """The product library; built in-tree when missing (never a fallback)."""
    from omnivoice_b200 import _native
    if not _native.LIB_PATH.exists():
        from omnivoice_b200 import build
        build.build()
    return _native.lib()


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import binding
    binding.oracle()
    return binding


@pytest.fixture(scope="session")
def decoding_golden():
    return json.loads((GOLDEN / "decoding_golden.json").read_text())


@pytest.fixture(scope="session")
def cuda_device():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.skip(f"needs sm_100 (B200), found sm_{major}{minor}")
    return torch.device("cuda:0")


def small_config(**kw):
    """A reduced-size model with the real kernel shapes (head_dim 128)."""
    from omnivoice_b200 import model_config
    base = dict(vocab_size=4096, hidden_size=256, intermediate_size=512, layers=2, heads=2,
                kv_heads=1)
    base.update(kw)
    return model_config(**base)


def oracle_config_from(cfg):
    from oracle import binding
    names = [f[0] for f in binding.OracleConfig._fields_]
    return binding.OracleConfig(**{n: getattr(cfg, n) for n in names})


os.environ.setdefault("OMNIVOICE_B200_TESTS", "1")


def guided_scores_f64(logits, frames, codebooks=8, vocab=1025, guidance=2.0):
    """The guided scores g = c + guidance (c - u) of every (frame, codebook)
    (c, u the conditional and unconditional log-softmax, generator_kernels.hip
    :212-265), in float64 from float32 logits [2F][codebooks * vocab];
    returns [codebooks][frames][vocab]."""
    import numpy as np
    x = logits.astype(np.float64).reshape(2, frames, codebooks, vocab)

    def lsm(a):
        m = a.max(axis=-1, keepdims=True)
        return a - (m + np.log(np.exp(a - m).sum(axis=-1, keepdims=True)))

    c, u = lsm(x[0]), lsm(x[1])
    return np.transpose(c + guidance * (c - u), (1, 0, 2))


def check_argmax_exact(pred, logits, frames, codebooks=8, vocab=1025, mask_id=1024,
                       guidance=2.0):
    """The predictions of identical logits must equal the argmax of the
    guided scores (lowest index on ties, the mask class excluded) wherever
    the top two scores are more than 16 float32 ulps apart.  Two
    implementations (the CUDA kernel, the oracle) may differ only inside
    that band: their float32 log-sum-exps differ in summation order and
    exponential, which shifts every score of a row by the same amount (no
    effect on the argmax), and then each score is rounded by a few
    operations of about half an ulp each.  Inside the band the prediction
    must still be one of the nearly tied indices; exact ties take the
    lowest index.  Returns (mismatches outside
    the band, items inside the band) after asserting the former is 0."""
    import numpy as np
    g = guided_scores_f64(logits, frames, codebooks, vocab, guidance)
    g[..., mask_id] = -np.inf
    top = g.max(axis=-1)
    best = g.argmax(axis=-1)
    second = np.partition(g, -2, axis=-1)[..., -2]
    ulp = np.exp2(np.floor(np.log2(np.abs(top))) - 23)
    band = 16 * ulp
    # Exact ties (equal float64 scores come from equal logits, which give
    # equal float32 scores in any implementation) take the lowest index.
    clear = ((top - second) > band) | (top == second)
    pred = np.asarray(pred).reshape(codebooks, frames)
    outside = int(((pred != best) & clear).sum())
    inside = int((~clear).sum())
    picked = np.take_along_axis(g, pred[..., None].astype(np.int64), axis=-1)[..., 0]
    bad_ties = int(((top - picked) > band)[~clear].sum())
    print(f"argmax: {outside} mismatches outside the tie band, {inside} near-ties "
          f"({int((pred != best).sum())} differ from the float64 argmax in total)")
    assert outside == 0
    assert bad_ties == 0
    return outside, inside

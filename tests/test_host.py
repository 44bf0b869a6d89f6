"""Host-side logic of the backend library, run on the CPU.

The shipped library (libnexus_cuda.so) must load here and export every
symbol of include/nexus_cuda.h; its host quantizers and GGUF writer are
checked byte-for-byte against the oracle.  No kernel is launched.
"""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
FORMATS = ["Q8_0", "Q4_0", "Q4_K", "Q2_K"]


def header_functions():
    text = (ROOT / "include" / "nexus_cuda.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nexus_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(nb):
    lib = nb._lib.load()
    names = header_functions()
    assert len(names) >= 25
    for n in names:
        assert hasattr(lib, n), n
    declared = {s[0] for s in nb._lib.SIGNATURES}
    assert set(names) == declared


def test_no_gpu_means_unavailable_not_fallback(nb):
    lib = nb._lib.load()
    caps = nb.cuda_capabilities()
    assert caps.backend == "cuda"
    if lib.nexus_cuda_is_available():
        pytest.skip("a GPU is present")
    assert caps.available is False
    h = C.c_void_p()
    rc = lib.nexus_cuda_backend_create(None, C.byref(h))
    assert rc == nb._lib.NEXUS_E_UNAVAILABLE and not h.value


def edge_inputs(rng, n):
    x = (rng.standard_normal(n) * 0.02).astype(np.float32)
    x[:256] = 0.0                     # all-zero super-block
    x[256:512] = 1.0                  # constant positive block (norm weights)
    x[512:768] = -0.5                 # constant negative block
    x[768:1024] = rng.standard_normal(256).astype(np.float32) * 1e-6  # tiny values
    x[1024:1280] = rng.standard_normal(256).astype(np.float32) * 3e4   # f16-range values
    return x


@pytest.mark.parametrize("fmt", FORMATS)
def test_host_quantizer_matches_oracle(nb, oracle, fmt):
    rng = np.random.default_rng(11)
    for n in (1, 31, 32, 255, 256, 300, 256 * 9 + 17):
        x = (rng.standard_normal(n) * 0.5).astype(np.float32)
        assert np.array_equal(nb.quantize_host(getattr(nb, fmt), x), oracle.quantize(getattr(oracle, fmt), x))
    x = edge_inputs(rng, 256 * 8)
    assert np.array_equal(nb.quantize_host(getattr(nb, fmt), x), oracle.quantize(getattr(oracle, fmt), x))


def test_format_bytes(nb, oracle):
    lib = nb._lib.load()
    for fmt in FORMATS:
        for n in (1, 32, 256, 300, 4096 * 14336):
            assert lib.nexus_format_bytes(getattr(nb, fmt), n) == oracle.type_size(getattr(oracle, fmt), n)


def test_synthetic_gguf_is_read_by_the_oracle(nb, oracle, tmp_path):
    cfg = dict(nb.CONFIGS["tiny"])
    path = tmp_path / "t.gguf"
    nb.write_synthetic_model(str(path), seed=3, threads=2, **cfg)
    m = oracle.Model(path)
    assert (m.info.num_layers, m.info.hidden_size, m.info.num_heads, m.info.num_kv_heads) == (4, 256, 8, 4)
    assert (m.info.head_dim, m.info.ff_dim, m.info.vocab_rows) == (32, 768, 4096)
    assert m.info.rope_freq_base == 10000.0 and m.info.max_seq_len == cfg["context_length"]
    # thread count of the generator does not change the file
    path2 = tmp_path / "t2.gguf"
    nb.write_synthetic_model(str(path2), seed=3, threads=5, **cfg)
    assert path.read_bytes() == path2.read_bytes()


def test_synthetic_weights_are_seeded_normal(nb, oracle, tmp_path):
    cfg = dict(nb.CONFIGS["tiny"], attn_format=nb.F32)
    path = tmp_path / "f32.gguf"
    nb.write_synthetic_model(str(path), seed=0, threads=2, **cfg)
    from tests.gguf_reader import read_tensor
    w = read_tensor(path, "blk.0.attn_q.weight")
    assert w.size == 256 * 256
    assert abs(float(w.mean())) < 1e-3 and abs(float(w.std()) - 0.02) < 5e-4


def test_bench_reference_arm_prints_one_contract_line():
    """`bench.py --impl reference` (the oracle port on the host cores) prints one
    JSON line with the contract's keys and the GPU arm's metric string, and
    never loads the CUDA library (its model file comes from the oracle's
    writer); the tiny config keeps it to seconds."""
    import json
    import subprocess
    import sys
    root = Path(__file__).resolve().parents[1]
    probe = ("import runpy, sys\n"
             "sys.argv = ['bench.py', '--impl', 'reference', '--config', 'tiny', '--steps', '2', '--warmup', '4']\n"
             "try:\n    runpy.run_path('bench.py', run_name='__main__')\nexcept SystemExit as e:\n    rc = e.code\n"
             "maps = open('/proc/self/maps').read()\n"
             "print('LOADED_CUDA_LIB' if 'libnexus_cuda' in maps else 'NO_CUDA_LIB')\n"
             "print('LOADED_ORACLE' if 'liboracle' in maps else 'NO_ORACLE')\n"
             "sys.exit(rc or 0)\n")
    r = subprocess.run([sys.executable, "-c", probe], capture_output=True, text=True, timeout=600, cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    assert "NO_CUDA_LIB" in r.stdout and "LOADED_ORACLE" in r.stdout, r.stdout
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "e2e", "cpu_baseline"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["warmup"] == 4
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["single_core"]["cores"] == 1 and d["cpu_baseline"]["single_core"]["value"] > 0
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    # the GPU arm prints the same metric string (the driver pairs the two lines by it)
    sys.path.insert(0, str(root))
    import bench
    assert d["metric"] == bench.METRIC
    src = (root / "bench.py").read_text()
    assert src.count('"metric": METRIC') == 2 and 'line["metric"]' not in src


def _write_tiny(model_dir):
    import os
    os.environ["NEXUS_MODEL_DIR"] = model_dir
    from nexus_b200.configs import model_path
    from oracle import oracle as O
    return str(model_path("tiny", writer=O.write_synthetic_model))


def test_model_path_concurrent_writers(tmp_path):
    """Ranks of a multi-GPU run may write the same synthetic model at once:
    each writes under its own temporary name and the renames leave one
    complete file (the run that found this raced on a shared name)."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    with ctx.Pool(3) as pool:
        paths = pool.map(_write_tiny, [str(tmp_path)] * 3)
    assert len(set(paths)) == 1
    files = sorted(p.name for p in tmp_path.iterdir())
    assert not [f for f in files if f.endswith(".tmp")], files
    from oracle import oracle as O
    m = O.Model(paths[0])
    assert m.info.num_layers == 4 and m.info.vocab_rows == 4096

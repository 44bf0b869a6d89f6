"""Model files the loader must refuse, through nexus_cuda_model_load.

The reference reads GGUF with io::Result errors (src/gguf/mod.rs:1091-1358)
and, when a tensor is unusable, silently falls back to a stateless decode
(src/engine/mod.rs:1160-1166).  The CUDA backend reports instead: a file cut
inside its header or its tensor data gives NEXUS_E_TRUNCATED, a wrong magic
NEXUS_E_INVALID, a missing file NEXUS_E_IO -- each with a message, nothing
left allocated -- and the same backend then loads the intact file and
decodes it exactly like the oracle."""
import shutil

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _load_error(nb, backend, path):
    eng = nb.InferenceEngine(backend)
    with pytest.raises(nb.NexusError) as err:
        eng.load_model(path)
    return err.value


def test_damaged_files_are_refused_and_the_backend_stays_usable(nb, oracle, tiny_path, tmp_path):
    from nexus_b200 import _lib as L
    data = open(tiny_path, "rb").read()
    be = nb.CudaBackend(device=0)
    free_before = be.memory_info().free_memory
    cases = {
        "tail": (data[:int(len(data) * 0.9)], L.NEXUS_E_TRUNCATED),   # tensor data cut short
        "header": (data[:40], L.NEXUS_E_TRUNCATED),                   # inside the metadata
        "magic": (b"GGUX" + data[4:], L.NEXUS_E_INVALID),
    }
    for name, (blob, code) in cases.items():
        p = tmp_path / f"{name}.gguf"
        p.write_bytes(blob)
        e = _load_error(nb, be, p)
        assert e.code == code, (name, e)
        assert str(e).split(":", 1)[1].strip(), name      # a message names the cause
    e = _load_error(nb, be, tmp_path / "missing.gguf")
    assert e.code == L.NEXUS_E_IO
    # nothing the refused loads allocated is still held (64 MB of slack for the allocator)
    assert be.memory_info().free_memory >= free_before - (64 << 20)
    # the same backend loads the intact file and matches the oracle
    good = tmp_path / "good.gguf"
    shutil.copy(tiny_path, good)
    eng = nb.InferenceEngine(be)
    eng.load_model(good)
    prompt = np.random.default_rng(8).integers(0, 4096, 12).tolist()
    assert eng.generate(prompt, 6) == oracle.Model(good).generate(prompt, 6)
    eng.close()
    be.close()

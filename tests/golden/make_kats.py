"""Write reference_kats.json: the known-answer tests of the reference's own
inline test modules (luen-eth/Nexus), transcribed from their source as data.

The reference is Rust and cannot be built here, so its golden values are
taken from the assertions in its tests.  Each entry names the test it comes
from (path:line in the reference project).  Run: python tests/golden/make_kats.py
"""
import json
import math
from pathlib import Path

KATS = {
    "q8_0_dequant": {
        "source": "src/gguf/mod.rs:1681-1695 test_q8_0_dequantization",
        "scale": 0.5, "q": [i - 16 for i in range(32)],
        "expect": {"0": -8.0, "16": 0.0, "31": 7.5},
    },
    "k_quant_sizes": {
        "source": "src/gguf/mod.rs:1697-1714 test_k_quant_dequantization; src/quant/mod.rs:1313-1339",
        "ramp": "i/31-4", "n": 300,
        "bytes": {"Q4_K": math.ceil(300 / 256) * 144, "Q2_K": math.ceil(300 / 256) * 84},
    },
    "roundtrip_bounds": {
        "source": "src/quant/mod.rs:1287-1352",
        "cases": [
            {"format": "Q8_0", "n": 64, "ramp": "i/16-2", "max_abs_err": 0.03},
            {"format": "Q4_0", "n": 64, "ramp": "i/16-2", "max_abs_err": 0.3},
            {"format": "Q4_K", "n": 300, "ramp": "i/31-4", "max_abs_err": 0.4},
            {"format": "Q2_K", "n": 300, "ramp": "i/31-4", "max_abs_err": 1.6},
        ],
    },
    "rms_norm": {
        "source": "src/kernel/mod.rs:288-301 test_rms_norm; src/backend/cpu.rs:201-217",
        "input": [1.0, 2.0, 3.0, 4.0], "weight": [1.0, 1.0, 1.0, 1.0], "eps": 1e-5,
        "expect_scale": "1/sqrt(30/4)", "tol": 1e-5,
    },
    "rope_pos0_identity": {
        "source": "src/kernel/mod.rs:277-286 test_rope",
        "input": [1.0, 2.0, 3.0, 4.0], "position": 0, "head_dim": 4, "base": 10000.0, "tol": 1e-5,
    },
    "packed_kv_roundtrip": {
        "source": "src/engine/mod.rs:1477-1494 test_quantized_kv_cache_roundtrip",
        "bits": 4, "head_dim": 8, "max_seq_len": 4,
        "key": [-1.0, -0.5, -0.25, 0.0, 0.25, 0.5, 0.75, 1.0],
        "value": [1.0, 0.75, 0.5, 0.25, 0.0, -0.25, -0.5, -1.0], "tol": 0.15,
    },
    "packed_kv_attention_finite": {
        "source": "src/engine/mod.rs:1496-1506 test_quantized_kv_attention_direct_path",
        "bits": 4, "head_dim": 2, "keys": [[1.0, 0.0], [0.0, 1.0]], "values": [[0.25, 0.75], [0.5, 0.5]],
        "q": [1.0, 0.0],
    },
    "greedy": {
        "source": "src/engine/mod.rs:1601-1610 test_greedy_sampling_picks_largest_logit",
        "logits": [0.1, 3.0, 1.0], "expect": 1,
    },
    "prefill_zero_layer": {
        "source": "src/engine/mod.rs:1700-1743 test_tiny_model_prefill_logits_are_stable",
        "token_embd": [1.0, 0.0, 0.0, 1.0], "output_norm": [1.0, 1.0], "output": [0.0, 0.0, 1.0, 0.0],
        "hidden": 2, "eps": 0.0, "tokens": [0], "expect": [0.0, math.sqrt(2.0)], "tol": 1e-6,
    },
    "decode_one_layer_shapes": {
        "source": "src/engine/mod.rs:1542-1599 test_decode_with_cache_runs_transformer_layer",
        "expect_logits_len": 6, "expect_seq_len": 1,
    },
    "kv_cache_shift": {
        "source": "src/engine/mod.rs:1526-1540 test_kv_cache_shift",
        "head_dim": 4, "max_seq_len": 3, "adds": 4, "expect_seq_len": 3,
    },
}

if __name__ == "__main__":
    out = Path(__file__).with_name("reference_kats.json")
    out.write_text(json.dumps(KATS, indent=1, sort_keys=True))
    print(out)

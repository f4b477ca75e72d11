"""Extract the plaintext golden values of the reference's sparse-MoE fixtures.

Reads the reference tree's committed fixtures (only the parts that do not need
the real checkpoint: deterministic input specs and their bf16 SHA-256, router
selections, bf16 logits and renormalised scores, route weights) and writes
reference_fixtures.json next to this script.  Run once in a container where
the reference tree is mounted:

    python tests/golden/make_golden.py /path/to/firewing

The known-answer values of the reference's unit tests are literals in
tests/test_oracle_golden.py, each citing its source line.
"""
import json
import os
import sys


def main(ref_root: str) -> None:
    fx = os.path.join(ref_root, "fixtures")
    router = json.load(open(os.path.join(fx, "router", "qwen3_8_flash_next_real.json")))
    expert = json.load(open(os.path.join(fx, "expert", "qwen3_8_flash_next_real.json")))
    mixture = json.load(open(os.path.join(fx, "mixture", "qwen3_8_flash_next_real.json")))
    sparse = json.load(open(os.path.join(fx, "sparse_moe", "qwen3_8_flash_next_layer0.json")))
    out = {
        "source": "x3haloed/firewing fixtures/{router,expert,mixture,sparse_moe} (plaintext fields only)",
        "hidden_size": router["configuration"]["hidden_size"],
        "num_experts": router["configuration"]["num_experts"],
        "top_k": router["configuration"]["top_k"],
        "router_cases": [
            {
                "name": c["name"],
                "layer": c["layer"],
                "input_spec": c["input_spec"],
                "input_bf16_sha256": c["input_bf16_sha256"],
                "selected_experts": c["selected_experts"],
                "selected_logits_bf16": c["selected_logits_bf16"],
                "normalized_scores_bf16": c["normalized_scores_bf16"],
            }
            for c in router["cases"]
        ],
        "expert_case": {
            "name": expert["case"]["name"],
            "expert": expert["case"]["expert"],
            "input_spec": expert["case"]["input_spec"],
            "input_bf16_sha256": expert["case"]["input_bf16_sha256"],
            "route_weight_bf16": expert["case"]["route_weight_bf16"],
        },
        "mixture_case": {
            "name": mixture["case"]["name"],
            "top_k_selection_order": mixture["case"]["top_k_selection_order"],
            "expert_execution_order": mixture["case"]["expert_execution_order"],
            "route_weights_bf16": {str(e["expert"]): e["route_weight_bf16"] for e in mixture["case"]["experts"]},
            "input_bf16_sha256": mixture["case"]["input_bf16_sha256"],
        },
        "sparse_moe_case": {
            "name": sparse["case"]["name"],
            "input_spec": sparse["case"]["input_spec"],
            "input_bf16_sha256": sparse["case"]["input_bf16_sha256"],
            "routed_mixture_sha256": sparse["case"]["expected_bf16_sha256"]["routed_mixture"],
        },
    }
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_fixtures.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
        f.write("\n")
    print("wrote", path)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <firewing source tree>")
    main(sys.argv[1])

"""Extracts the MoE layer of the reference's DeepSeek-V4 tiny fixture into
deepseek_v4_tiny_moe.json (beside this script).

The reference's tests/fixtures/deepseek_v4_tiny_oracle.json (written by its
tools/generate_deepseek_v4_tiny_oracle.py, replayed by the reference test
independent_tiny_oracle_matches_one_hash_moe_layer, src/models/deepseek_v4/runtime.rs:4603-4646)
holds a one-layer, one-token DeepSeek-V4 model.  Only the routed-expert part is kept: the FFN
input, the F32 router, the token's hash experts, the three F32 routed experts and the shared
expert, and the expected router logits, routes, per-route expert outputs, shared expert output
and MoE branch.

    python tests/golden/make_deepseek_v4_tiny_moe.py <reference checkout>/tests/fixtures/deepseek_v4_tiny_oracle.json
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main(src):
    d = json.load(open(src))
    geo, w, exp = d["geometry"], d["weights"], d["expected"]
    token, top_k = d["token"], geo["num_experts_per_tok"]
    tid2eid = w["layers.0.ffn.gate.tid2eid"]["values"]

    def mat(name):
        t = w[name]
        assert t["dtype"] == "F32", name
        return {"shape": t["shape"], "values": t["values"]}

    out = {
        "source": "reference tests/fixtures/deepseek_v4_tiny_oracle.json (format_version %d)"
                  % d["format_version"],
        "hidden": geo["hidden_size"], "intermediate": geo["moe_intermediate_size"],
        "experts": geo["n_routed_experts"], "top_k": top_k,
        "routed_scaling_factor": geo["routed_scaling_factor"],
        "swiglu_limit": geo["swiglu_limit"],
        "hash_experts": tid2eid[token * top_k:(token + 1) * top_k],
        "router": mat("layers.0.ffn.gate.weight"),
        "routed": [{p: mat("layers.0.ffn.experts.%d.%s.weight" % (e, p)) for p in ("w1", "w2", "w3")}
                   for e in range(geo["n_routed_experts"])],
        "shared": {p: mat("layers.0.ffn.shared_experts.%s.weight" % p) for p in ("w1", "w2", "w3")},
        "ffn_input": exp["ffn_input"],
        "expected": {k: exp[k] for k in ("router_logits", "routes", "routed_experts",
                                         "shared_expert", "moe_branch")},
    }
    dst = os.path.join(HERE, "deepseek_v4_tiny_moe.json")
    with open(dst, "w") as f:
        json.dump(out, f, indent=1)
    print(dst)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(sys.argv[1])

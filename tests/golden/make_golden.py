"""Copies the reference's golden logits into compact fixtures.

Source: krikil-rs test_reference_logits.json (18-token prompt -> last-token
logits) and test_reference_step_logits.json (the same prompt + token 199 ->
logits), the vectors src/model.rs:791-932 checks at max-abs 1e-4.  They were
produced by PyTorch on the real Pebble-25M checkpoint, which is not available
here, so tests use them only when KRIKIL_PEBBLE_WEIGHTS names that checkpoint.

Run:  python tests/golden/make_golden.py /path/to/krikil-rs
"""
import json
import os
import sys


def main(ref_dir: str) -> None:
    here = os.path.dirname(os.path.abspath(__file__))
    for src, dst in (("test_reference_logits.json", "reference_prefill_logits.json"),
                     ("test_reference_step_logits.json", "reference_step_logits.json")):
        with open(os.path.join(ref_dir, src)) as f:
            d = json.load(f)
        out = {"source": src, "tokens": d["tokens"], "logits": d["logits"]}
        if "step_token" in d:
            out["step_token"] = d["step_token"]
        with open(os.path.join(here, dst), "w") as f:
            json.dump(out, f, separators=(",", ":"))
        print("wrote", dst, len(out["logits"]), "logits")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {os.path.basename(__file__)} <krikil-rs checkout>")
    main(sys.argv[1])

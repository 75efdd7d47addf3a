"""Golden manifest: the reference's own manifest builder (``tools/k3_manifest.py build``)
run over the tiny checkpoint of ``tests/ckpt_util.py`` (seed 0). Needs the reference
tree (read only); run here, not on the GPU box:

    python tests/golden/make_manifest_golden.py --ref /path/to/reference

Writes ``tests/golden/manifest_tiny.json``: the meta record (minus the machine-specific
checkpoint path) and every tensor record, in the builder's order.
"""
import json
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))


def main(ref: str) -> None:
    import ckpt_util
    sys.path.insert(0, str(Path(ref) / "tools"))
    import k3_manifest
    with tempfile.TemporaryDirectory() as td:
        ck = Path(td) / "ckpt"
        ckpt_util.make_tiny_k3(ck, seed=0)
        k3_manifest.set_ckpt(ck)
        out = Path(td) / "manifest.jsonl.gz"
        k3_manifest.build(out)
        meta, recs = k3_manifest.load_manifest(out)
    meta.pop("checkpoint")
    (HERE / "manifest_tiny.json").write_text(json.dumps({"meta": meta, "records": recs}, indent=0))
    print(f"{len(recs)} records")


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", type=Path, required=True, help="reference checkout (read-only)")
    main(str(ap.parse_args().ref))

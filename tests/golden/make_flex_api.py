"""Records the public API of the reference's flex_gemm operator package (promptmoge/_fallback/flex_gemm) as
tests/golden/flex_gemm_api.json: every module-level name, the constructor and forward signatures of the nn classes,
the function signatures of ops, and NeighborCache's public attributes.  tests/test_flex_gemm_api.py compares the
drop-in package promptmoge_b200.flex_gemm against it.

    python tests/golden/make_flex_api.py /path/to/reference/promptmoge/_fallback
"""
import inspect
import json
import sys
from pathlib import Path


def sig(fn):
    out = []
    for p in inspect.signature(fn).parameters.values():
        d = None if p.default is inspect.Parameter.empty else repr(p.default)
        out.append([p.name, p.kind.name, d])
    return out


def main(fallback_dir: str) -> None:
    sys.path.insert(0, fallback_dir)
    import flex_gemm
    from flex_gemm import nn as fnn, ops as fops
    api = {"nn": {}, "ops": {}, "nn_all": list(fnn.__all__), "ops_all": list(fops.__all__)}
    for name in fnn.__all__:
        cls = getattr(fnn, name)
        api["nn"][name] = {"init": sig(cls.__init__), "forward": sig(cls.forward)}
    for name in fops.__all__:
        obj = getattr(fops, name)
        if inspect.isclass(obj):
            api["ops"][name] = {"class": True, "init": sig(obj.__init__),
                                "members": sorted(n for n in dir(obj) if not n.startswith("_"))}
        else:
            api["ops"][name] = {"class": False, "sig": sig(obj)}
    out = Path(__file__).with_name("flex_gemm_api.json")
    out.write_text(json.dumps(api, indent=1, sort_keys=True))
    print("wrote", out, flex_gemm.__version__)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} /path/to/PromptMoGe/promptmoge/_fallback")
    main(sys.argv[1])

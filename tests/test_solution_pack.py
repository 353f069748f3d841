"""The flashinfer-bench packaging: solution.json has the harness schema and
its embedded main.py exposes the package's run() (loaded as the harness's
PythonBuilder would, from the source text)."""
import importlib.util
import json

from rocm_flashinfer_contest_b200 import gdn_decode, gdn_prefill
from rocm_flashinfer_contest_b200.solution import pack


def test_pack_writes_harness_schema(tmp_path):
    paths = pack.pack(str(tmp_path))
    assert len(paths) == 2
    for path, (definition, name, _) in zip(paths, pack.SOLUTIONS):
        sol = json.load(open(path))
        assert sol["definition"] == definition and sol["name"] == name
        spec = sol["spec"]
        assert spec["language"] == "python" and spec["entry_point"] == "main.py::run"
        assert spec["destination_passing_style"] is False
        assert [s["path"] for s in sol["sources"]] == ["main.py"]


def test_embedded_main_exposes_run(tmp_path):
    paths = pack.pack(str(tmp_path))
    expect = [gdn_decode.run, gdn_prefill.run]
    for path, fn in zip(paths, expect):
        src = json.load(open(path))["sources"][0]["content"]
        main = tmp_path / f"main_{fn.__module__.split('.')[-1]}.py"
        main.write_text(src)
        spec = importlib.util.spec_from_file_location(main.stem, main)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        assert mod.run is fn

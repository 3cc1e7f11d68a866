"""The documentation names only what exists: every function and method in the
API reference's tables, and every server flag the README and the deployment
guide mention, are checked against the code."""
import importlib
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = "3080_mod_p2p_sglang_patch_b200"


def _read(rel):
    with open(os.path.join(ROOT, rel)) as f:
        return f.read()


def _section(text, start, end=None):
    i = text.index(start)
    j = text.index(end, i) if end else len(text)
    return text[i:j]


def _called_names(text):
    """Names written as `name(` or `Class.name(` at the start of a table cell
    or of a list in one (the signatures the tables document, not formulas in
    their descriptions)."""
    return set(re.findall(r"(?:^\| |, )`(?:[A-Za-z_]+\.)?([A-Za-z_][A-Za-z0-9_]*)\(", text, re.M))


def test_api_reference_names_exist():
    doc = _read("docs/api.md")
    par = importlib.import_module(f"{PKG}.parallel")
    ops = importlib.import_module(f"{PKG}.ops")
    eng = importlib.import_module(f"{PKG}.engine")
    comm = _section(doc, "### `MailboxAR(", "### `CommConfig`")
    missing = [n for n in _called_names(comm) if n != "MailboxAR" and not hasattr(par.MailboxAR, n)]
    kern = _section(doc, "## Kernels", "## Engine")
    missing += [f"ops.{n}" for n in _called_names(kern) if not hasattr(ops, n)]
    engine = _section(doc, "## Engine", "## Server")
    missing += [f"LLMEngine.{n}" for n in _called_names(engine)
                if n not in ("LLMEngine", "SamplingParams") and not hasattr(eng.LLMEngine, n)
                and n not in ("llama_8b", "llama_70b", "tiny")]
    cfg = importlib.import_module(f"{PKG}.config").CommConfig()
    fields = set(re.findall(r"^\| `([a-z_]+)`", _section(doc, "### `CommConfig`", "### `TPGroup"), re.M))
    fields |= {f for row in re.findall(r"^\| (`[a-z_]+`(?:, `[a-z_]+`)+) \|", doc, re.M)
               for f in re.findall(r"`([a-z_]+)`", row)} & set(vars(cfg))
    missing += [f"CommConfig.{f}" for f in fields if not hasattr(cfg, f)]
    models = importlib.import_module(f"{PKG}.models")
    missing += [f"LlamaConfig.{n}" for n in ("llama_8b", "llama_70b", "tiny") if not hasattr(models.LlamaConfig, n)]
    assert not missing, missing


def test_documented_server_flags_parse():
    cli = importlib.import_module(f"{PKG}.server.cli")
    p = cli.build_parser()
    known = {s for a in p._actions for s in a.option_strings}
    text = _section(_read("README.md"), "## Server", "## Examples") + _read("docs/deploy.md")
    flags = set(re.findall(r"(?<![\w-])(--[a-z][a-z0-9-]+)", text))
    launcher = {"--nproc-per-node", "--master-addr", "--nnodes", "--master-port", "--backends"}
    missing = sorted(f for f in flags - launcher if f not in known)
    assert not missing, missing

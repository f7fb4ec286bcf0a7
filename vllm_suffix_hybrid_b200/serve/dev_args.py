"""Dev-mode command-line splice for the server (SUFFIX_HYBRID_DEV_ARGS=1; production never sets it).

When enabled and the file SUFFIX_HYBRID_DEV_ARGS_FILE (default ./dev_args.json) exists, its entries are
merged into the server's argv before parsing, then the file is renamed to <name>.last.json so every
start applies one reviewed delta.  Entry forms, a JSON list (the reference's format, dev_args.py:1-20):

  "--flag"              bare flag, appended when absent
  ["--flag", "value"]   flag with a value; replaces the first occurrence in place (others are removed)
  ["--flag", null]      removes every occurrence

Flags that select the model (--model, --served-model-name, -m) can not be spliced.
"""
from __future__ import annotations

import json
import os
from typing import List, Optional

RESERVED = frozenset({"--model", "--model-path", "-m", "--served-model-name"})


def _groups(argv: List[str]) -> List[List[str]]:
    """argv as [flag, value?] / [positional] groups in order; --flag=value stays one token."""
    groups: List[List[str]] = []
    for tok in argv:
        prev = groups[-1] if groups else None
        takes_value = (prev is not None and prev[0].startswith("--") and "=" not in prev[0] and len(prev) == 1)
        if not tok.startswith("--") and takes_value:
            prev.append(tok)
        else:
            groups.append([tok])
    return groups


def _name(group: List[str]) -> Optional[str]:
    return group[0].split("=", 1)[0] if group[0].startswith("--") else None


def splice(argv: List[str], entries) -> List[str]:
    groups = _groups(list(argv))
    for entry in entries:
        if isinstance(entry, str):
            flag, value, remove = entry, None, False
        elif isinstance(entry, list) and len(entry) == 2 and isinstance(entry[0], str):
            flag, value, remove = entry[0], entry[1], entry[1] is None
        else:
            raise ValueError(f"dev args entry must be \"--flag\" or [\"--flag\", value|null]: {entry!r}")
        if not flag.startswith("--"):
            raise ValueError(f"dev args flag must start with --: {flag!r}")
        if flag in RESERVED:
            raise ValueError(f"dev args may not change {flag}")
        hits = [i for i, g in enumerate(groups) if _name(g) == flag]
        if remove:
            groups = [g for g in groups if _name(g) != flag]
            continue
        new = [flag] if value is None else [flag, str(value)]
        if hits:
            groups[hits[0]] = new
            groups = [g for i, g in enumerate(groups) if i not in hits[1:]]
        else:
            groups.append(new)
    return [tok for g in groups for tok in g]


def apply(argv: List[str], path: Optional[str] = None) -> Optional[list]:
    """Splice the dev args file into argv (in place); returns the applied entries or None."""
    if os.environ.get("SUFFIX_HYBRID_DEV_ARGS", "").strip() != "1":
        return None
    path = path or os.environ.get("SUFFIX_HYBRID_DEV_ARGS_FILE", "dev_args.json")
    if not os.path.exists(path):
        return None
    with open(path) as fh:
        entries = json.load(fh)
    if not isinstance(entries, list):
        raise ValueError(f"{path}: expected a JSON list")
    argv[:] = splice(argv, entries)
    root, _ = os.path.splitext(path)
    os.replace(path, root + ".last.json")
    return entries

"""Small JSON helpers for result artifacts (atomic writes, object reads).

Same contract as the reference's ``src/tklab/harness/jsonio.py``: a result
file is either absent or a complete JSON object, never a torn write.
"""

from __future__ import annotations

import json
import os
import tempfile
from pathlib import Path
from typing import Any, TypeAlias

JsonObject: TypeAlias = dict[str, Any]


def write_json_atomic(path: Path, payload: JsonObject) -> None:
    """Write ``payload`` as indented JSON to ``path`` through a same-directory rename."""
    path.parent.mkdir(parents=True, exist_ok=True)
    fd, tmp_name = tempfile.mkstemp(prefix=f".{path.name}.", suffix=".tmp", dir=path.parent)
    try:
        with os.fdopen(fd, "w", encoding="utf-8") as handle:
            json.dump(payload, handle, indent=2, sort_keys=False)
            handle.write("\n")
        os.replace(tmp_name, path)
    except BaseException:
        Path(tmp_name).unlink(missing_ok=True)
        raise


def read_json_object(path: Path) -> JsonObject:
    """Read a JSON file whose top level must be an object."""
    payload = json.loads(path.read_text(encoding="utf-8"))
    if not isinstance(payload, dict):
        raise ValueError(f"{path}: expected a JSON object")
    return payload

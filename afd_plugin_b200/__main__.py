"""``python -m afd_plugin_b200 <command> ...`` (also installed as ``afd-b200``).

Commands: ``serve`` (completions server), ``proxy`` (load-balancing /
prefill-decode proxy), ``serve-bench`` (online load benchmark), ``e2e``
(scenario runner), ``gsm8k`` (accuracy against a server), ``launch`` (local
multi-process AFD run).
"""

from __future__ import annotations

import importlib
import sys

COMMANDS = {
    "serve": ("afd_plugin_b200.serving.__main__", "main"),
    "proxy": ("afd_plugin_b200.serving.proxy", "main"),
    "serve-bench": ("afd_plugin_b200.bench.serve_bench", "main"),
    "e2e": ("afd_plugin_b200.e2e.runner", "main"),
    "gsm8k": ("afd_plugin_b200.e2e.gsm8k", "main"),
    "launch": ("afd_plugin_b200.runtime.launcher", "main"),
}


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv or argv[0] in ("-h", "--help") or argv[0] not in COMMANDS:
        print(__doc__.strip())
        return 0 if argv and argv[0] in ("-h", "--help") else 2
    module, fn = COMMANDS[argv[0]]
    rc = getattr(importlib.import_module(module), fn)(argv[1:])
    return rc if isinstance(rc, int) else 0


if __name__ == "__main__":
    sys.exit(main())

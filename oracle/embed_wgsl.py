"""Writes bllm/shaders_generated.h for compiling the reference's launchers in
place — TEST AND INTEGRATION BUILD INFRASTRUCTURE ONLY.

The reference's launchers (src/core/kernels/*/*.cpp) include a header its
build generates: every WGSL source of the project as an inline constexpr
std::string_view named by the file's stem, in namespace bllm::shaders. This
script writes the same declarations from the .wgsl files where they lie
(nothing is copied into this repository; the output goes under a build
folder): the launchers compare a launch's kernel text against these views,
so a shim compiled against the same header can tell the kernels apart.

    python embed_wgsl.py <reference root> <output header>
"""
from __future__ import annotations

import os
import sys

DELIMITER = "CBWGSL"


def sources(root: str) -> list[str]:
    out = []
    for base, _, files in os.walk(os.path.join(root, "src")):
        out += [os.path.join(base, f) for f in files if f.endswith(".wgsl")]
    return sorted(out, key=os.path.basename)


def render(root: str) -> str:
    lines = ["// Written by embed_wgsl.py from the reference's WGSL sources. Do not edit.", "#pragma once", "",
             "#include <string_view>", "", "namespace bllm::shaders {", ""]
    seen = set()
    for path in sources(root):
        name = os.path.splitext(os.path.basename(path))[0]
        if name in seen:
            raise SystemExit(f"two WGSL sources named {name}")
        seen.add(name)
        with open(path, encoding="utf-8") as fh:
            text = fh.read()
        if f"){DELIMITER}\"" in text:
            raise SystemExit(f"{path} holds the raw-string delimiter")
        lines.append(f'inline constexpr std::string_view {name} = R"{DELIMITER}({text}){DELIMITER}";')
        lines.append("")
    lines.append("}  // namespace bllm::shaders")
    return "\n".join(lines) + "\n"


def main() -> None:
    root, out = sys.argv[1], sys.argv[2]
    text = render(root)
    os.makedirs(os.path.dirname(out), exist_ok=True)
    if os.path.exists(out):
        with open(out, encoding="utf-8") as fh:
            if fh.read() == text:
                return
    with open(out, "w", encoding="utf-8") as fh:
        fh.write(text)


if __name__ == "__main__":
    main()

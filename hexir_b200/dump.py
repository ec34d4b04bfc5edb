"""Print the contents of a .hxb module: python -m hexir_b200.dump FILE [...]

The module's header, sections, entry points with their command lists,
executables (kernel kinds including the fused ones, image extents) and the
LAUNCH records that say which GPUs run each executable.  It reads the bytes
with the Python reader in hexir_b200.api, independently of the C loader,
and needs no GPU.  The reference's tools/hxb-dump.py knows the four base
sections; this one also decodes the LAUNCH section (kind 5) and kernel kinds
4-6.
"""

import struct
import sys

from . import api

SECTION_NAMES = {1: "SYMBOLS", 2: "PROGRAM", 3: "RODATA", 4: "EXECUTABLES",
                 5: "LAUNCH"}
KERNEL_KINDS = {1: "matmul", 2: "add", 3: "relu", 4: "matmul_relu",
                5: "matmul_add", 6: "matmul_add_relu", 7: "leaky_relu",
                8: "elu", 9: "sigmoid", 10: "tanh", 11: "softmax", 12: "gelu",
                13: "swish", 14: "mish"}
COMMANDS = {0: "END", 1: "ALLOC", 2: "CONST", 3: "DISPATCH", 4: "PRINT"}


def entry_names(blob: bytes) -> list:
    sections = api.read_sections(blob)
    off, size = sections[1]
    names = []
    for i in range(size // api.SYMBOL.size):
        name, _pc, _ = api.SYMBOL.unpack_from(blob, off + i * api.SYMBOL.size)
        names.append(name.rstrip(b"\0").decode())
    return names


def format_command(kind: int, ops: tuple, exes: list) -> str:
    name = COMMANDS.get(kind, f"kind{kind}")
    if kind == 1:
        return f"ALLOC    slot {ops[0]} bytes {ops[1]}"
    if kind == 2:
        return f"CONST    slot {ops[0]} rodata +{ops[1]} bytes {ops[2]}"
    if kind == 3:
        exe = exes[ops[0]].name if ops[0] < len(exes) else "?"
        args = " ".join(str(x) for x in ops[2:-1])
        return f"DISPATCH {exe} ({args}) -> slot {ops[-1]}"
    if kind == 4:
        return f"PRINT    slot {ops[0]} {ops[1]}x{ops[2]}"
    return name


def dump(blob: bytes, out=sys.stdout) -> None:
    if len(blob) < api.HEADER.size or blob[:8] != b"HEXIRMOD":
        raise ValueError("not a version 3 hexir module")
    api.read_sections(blob)  # checks the version and the section table
    magic, version, flags, count, _ = api.HEADER.unpack_from(blob, 0)
    print(f"module: {magic.decode(errors='replace')} v{version} flags={flags} "
          f"{count} sections, {len(blob)} bytes", file=out)
    for i in range(count):
        kind, _f, off, size = api.SECTION.unpack_from(
            blob, api.HEADER.size + i * api.SECTION.size)
        print(f"  section {SECTION_NAMES.get(kind, f'kind {kind}'):<12} "
              f"offset {off:>10} size {size}", file=out)
    exes = api.read_executables(blob)
    launch = api.read_launch(blob)
    print(f"executables: {len(exes)}", file=out)
    for i, e in enumerate(exes):
        where = "cuda" if e.device == 1 else "cpu"
        if i < len(launch) and launch[i].abi:
            first, n = launch[i].device_first, launch[i].device_count
            where = f"cuda:{first}" if n <= 1 else f"cuda:{first}-{first + n - 1}"
        dims = f"{e.m}x{e.n}" + (f"x{e.k}" if e.k else "")
        image = (f"image +{e.image_offset} ({e.image_size} B)" if e.image_size
                 else "descriptor")
        print(f"  [{i}] {e.name:<16} {KERNEL_KINDS.get(e.kind, f'kind {e.kind}'):<16} "
              f"{where:<10} {dims:<18} {image}", file=out)
    for name in entry_names(blob):
        cmds = api.read_program(blob, name)
        print(f"entry {name}: {len(cmds)} commands", file=out)
        for kind, ops in cmds:
            print("  " + format_command(kind, ops, exes), file=out)


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    if not argv:
        print(__doc__.strip().splitlines()[0], file=sys.stderr)
        return 2
    status = 0
    for path in argv:
        try:
            with open(path, "rb") as f:
                blob = f.read()
            dump(blob)
        except (OSError, ValueError, KeyError, struct.error) as err:
            print(f"{path}: {err}", file=sys.stderr)
            status = 1
    return status


if __name__ == "__main__":
    sys.exit(main())

#!/usr/bin/env bash
# Installs the unmodified reference package (msda_triton: ops.py, kernels.py,
# metal.py) into baseline/_ref for bench.py's GPU-bar leg, which times the
# reference's own Triton kernels on the same B200.
#
#   MSDA_REFERENCE=<path to the reference checkout> baseline/install_reference.sh
#
# First the plain offline pip install. The reference builds with `uv_build`,
# which the offline wheelhouse does not carry; when that fails, the same
# install runs from a copy under /tmp whose [build-system] table names
# setuptools instead (package code untouched: only the packaging backend
# differs). baseline/_ref is git-ignored and travels with the repository
# snapshot to the GPU box.
set -euo pipefail
here="$(cd "$(dirname "$0")" && pwd)"
ref="${MSDA_REFERENCE:?set MSDA_REFERENCE to the reference checkout}"
target="$here/_ref"
rm -rf "$target"
pip_args=(--no-index --no-build-isolation --find-links /opt/wheelhouse --target "$target")
if python -m pip install "${pip_args[@]}" "$ref" >/dev/null 2>&1; then
  echo "installed $ref into $target (pip, stock build backend)"
  exit 0
fi
tmp="$(mktemp -d /tmp/msda_ref_src.XXXXXX)"
cp -r "$ref/src" "$ref/pyproject.toml" "$ref/README.md" "$ref/LICENSE" "$tmp/"
python - "$tmp/pyproject.toml" <<'PY'
import re, sys
p = sys.argv[1]
t = open(p).read()
t = re.sub(r"\[build-system\][^\[]*",
           '[build-system]\nrequires = ["setuptools"]\nbuild-backend = "setuptools.build_meta"\n\n', t, count=1)
t += '\n[tool.setuptools.packages.find]\nwhere = ["src"]\n'
open(p, "w").write(t)
PY
python -m pip install "${pip_args[@]}" --no-deps "$tmp" >/dev/null
rm -rf "$tmp"
echo "installed $ref into $target (pip --no-deps, setuptools backend on a /tmp copy)"

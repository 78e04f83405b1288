#!/usr/bin/env bash
# Installs the reference implementation, unmodified, into baseline/_ref (the
# "beat this" GPU ops and the reference's own CPU path for bench.py and
# tests/test_reference_gpu.py). One offline pip install per sub-project, from a
# temporary copy because setuptools writes build files next to the sources:
#   triton/ -> package fds_triton        (Triton kernels, TritonModel, TritonPipeline)
#   trt/    -> package fastdialoguesidon (flexrel_triton.torch_core_chunked, the fp32 CPU path)
# --no-deps: torch, triton and transformers come from the image; the trt
# project pins tensorrt / onnx wheels that are not installed (the modules used
# here do not import them).
# Usage: baseline/install_ref.sh <reference checkout>
set -euo pipefail
src="${1:?usage: $0 <reference checkout>}"
here="$(cd "$(dirname "$0")" && pwd)"
tmp="$(mktemp -d)"
trap 'rm -rf "$tmp"' EXIT
for sub in triton trt; do
    cp -r "$src/$sub" "$tmp/$sub"
    python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
        --target "$here/_ref" --upgrade "$tmp/$sub"
done

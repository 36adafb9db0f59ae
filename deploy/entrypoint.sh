#!/usr/bin/env bash
# Container entrypoint for one B200 node: optional code overlay, a check that the
# in-tree extension matches the sources, then one serving rank per visible GPU.
#
# Environment:
#   CODE_TGZ        optional path or http(s) URL of a code tarball extracted over /app
#                   (a code change without an image rebuild; the extension is rebuilt)
#   NGPU            ranks to start (default: every visible GPU)
#   PORT            HTTP port of rank 0 (default 8000)
#   NCCL_NVLS_ENABLE  left to NCCL's default (NVLink SHARP on) unless set
# Arguments are passed to the server (``python -m dsv4_flash_deployment_b200.serving``).
set -euo pipefail
cd /app

if [[ -n "${CODE_TGZ:-}" ]]; then
  if [[ "$CODE_TGZ" == http://* || "$CODE_TGZ" == https://* ]]; then
    curl -fsSL "$CODE_TGZ" | tar -xz -C /app
  else
    tar -xzf "$CODE_TGZ" -C /app
  fi
  echo "entrypoint: overlaid code from $CODE_TGZ" >&2
  python -c "import __graft_entry__ as g; g.build()"
fi

NGPU="${NGPU:-$(nvidia-smi --query-gpu=index --format=csv,noheader | wc -l)}"
PORT="${PORT:-8000}"
echo "entrypoint: host=$(hostname) gpus=${NGPU} port=${PORT}" >&2
nvidia-smi --query-gpu=index,name,memory.total,clocks.max.sm --format=csv >&2 || true

if [[ "$NGPU" -le 1 ]]; then
  exec python -m dsv4_flash_deployment_b200.serving --host 0.0.0.0 --port "$PORT" "$@"
fi
exec python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NGPU" --master-addr 127.0.0.1 \
    --master-port "${MASTER_PORT:-29500}" -m dsv4_flash_deployment_b200.serving --host 0.0.0.0 --port "$PORT" "$@"

#!/usr/bin/env bash
# Start a job across hosts: one process per rank, ranks listed in a host file.
#
#   examples/launch_multinode.sh hosts.txt examples/multinode_allreduce.py [script args...]
#
# hosts.txt, one entry per line, in rank order ('#' comments allowed):
#
#   10.0.0.1:29500        one rank on this host, listening on port 29500
#   10.0.0.2:29500:4      four ranks on this host, ports 29500..29503,
#                         LOCAL_RANK 0..3 (one GPU each with --device cuda)
#
# Every process gets RANK, WORLD_SIZE, LOCAL_RANK and MINI_NCCL_HOSTS (the
# full rank -> host:port list), which is all init_process_group() needs.
# Processes on the first host run locally (their output stays in this
# terminal); the others are started over ssh (passwordless, BatchMode) in
# REMOTE_DIR (default: this directory).  If any rank fails, the processes
# this script started are stopped and its exit status is returned.
# (Same contract as the reference's scripts/launch_multinode.sh; GPU ranks
# on one host also share peer memory through the device communicator.)
set -euo pipefail

HOSTFILE=${1:?usage: launch_multinode.sh <hostfile> <script> [args...]}
SCRIPT=${2:?usage: launch_multinode.sh <hostfile> <script> [args...]}
shift 2
REMOTE_DIR=${REMOTE_DIR:-$(pwd)}
PYTHON=${PYTHON:-python}

hosts=() ports=() locals=()
first_host=""
while read -r line; do
  line=${line%%#*}
  line=$(echo "$line" | tr -d '[:space:]')
  [[ -z "$line" ]] && continue
  IFS=: read -r h p n <<< "$line"
  p=${p:-29500}
  n=${n:-1}
  [[ -z "$first_host" ]] && first_host=$h
  for ((i = 0; i < n; i++)); do
    hosts+=("$h") ports+=($((p + i))) locals+=("$i")
  done
done < "$HOSTFILE"

WORLD_SIZE=${#hosts[@]}
(( WORLD_SIZE > 0 )) || { echo "no ranks in $HOSTFILE" >&2; exit 2; }
entries=()
for ((r = 0; r < WORLD_SIZE; r++)); do entries+=("${hosts[$r]}:${ports[$r]}"); done
MINI_NCCL_HOSTS=$(IFS=,; echo "${entries[*]}")
echo "world_size=$WORLD_SIZE hosts=$MINI_NCCL_HOSTS"

pids=()
stop_all() {
  for pid in "${pids[@]}"; do kill "$pid" 2>/dev/null || true; done
}
trap stop_all INT TERM

quoted_args=$(printf '%q ' "$@")
for ((r = 0; r < WORLD_SIZE; r++)); do
  vars="MINI_NCCL_HOSTS=$MINI_NCCL_HOSTS WORLD_SIZE=$WORLD_SIZE RANK=$r LOCAL_RANK=${locals[$r]}"
  if [[ "${hosts[$r]}" == "$first_host" ]]; then
    env MINI_NCCL_HOSTS="$MINI_NCCL_HOSTS" WORLD_SIZE="$WORLD_SIZE" RANK="$r" LOCAL_RANK="${locals[$r]}" \
      "$PYTHON" "$SCRIPT" "$@" &
  else
    ssh -o BatchMode=yes "${hosts[$r]}" "cd $(printf '%q' "$REMOTE_DIR") && $vars $PYTHON $(printf '%q' "$SCRIPT") $quoted_args" &
  fi
  pids+=($!)
done

status=0
for pid in "${pids[@]}"; do
  if ! wait "$pid"; then
    status=$?
    stop_all
  fi
done
exit "$status"

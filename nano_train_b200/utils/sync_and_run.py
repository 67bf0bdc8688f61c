"""Development workflow: publish the working tree, then pull and run it on a remote machine.

    python -m nano_train_b200.utils.sync_and_run [--message MSG] [--no-push]
        [--remote user@host] [--remote-dir DIR] [--command CMD] [--dry-run]

Steps (each printed before it runs; ``--dry-run`` prints them only):
1. if the tree has changes, ``git add -A`` and ``git commit -m MSG`` (default: a timestamped message);
2. ``git push`` of the current branch (skipped with ``--no-push``);
3. the remote side: ``cd DIR && git pull --ff-only && CMD``. With ``--remote`` it runs over ``ssh``;
   without it the lines are printed as a notebook cell to paste into the remote notebook (the
   reference's script writes the same kind of Colab cell, scripts/sync_and_run.sh:110-184).

Returns non-zero as soon as a step fails; nothing is retried.
"""
from __future__ import annotations

import argparse
import datetime
import shlex
import subprocess
import sys
from typing import Optional


def _git(args: list[str], cwd: Optional[str]) -> subprocess.CompletedProcess:
    return subprocess.run(["git", *args], cwd=cwd, capture_output=True, text=True)


def plan(*, cwd: Optional[str] = None, message: Optional[str] = None, push: bool = True,
         remote: Optional[str] = None, remote_dir: str = "nano-train-b200",
         command: str = "python -m pytest tests -m 'not gpu' -q") -> list[list[str]]:
    """The commands the workflow would run, as argv lists, given the current state of the tree."""
    steps: list[list[str]] = []
    if _git(["status", "--porcelain"], cwd).stdout.strip():
        msg = message or f"sync {datetime.datetime.now():%Y-%m-%d %H:%M:%S}"
        steps += [["git", "add", "-A"], ["git", "commit", "-m", msg]]
    if push:
        steps.append(["git", "push"])
    remote_cmd = f"cd {shlex.quote(remote_dir)} && git pull --ff-only && {command}"
    if remote:
        steps.append(["ssh", remote, remote_cmd])
    return steps


def notebook_cell(remote_dir: str, command: str, repo_url: Optional[str]) -> str:
    clone = f"!test -d {shlex.quote(remote_dir)} || git clone {repo_url} {shlex.quote(remote_dir)}\n" if repo_url else ""
    return f"{clone}%cd {remote_dir}\n!git pull --ff-only\n!{command}\n"


def main(argv: Optional[list[str]] = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--message", default=None)
    ap.add_argument("--no-push", action="store_true")
    ap.add_argument("--remote", default=None, help="user@host to run on over ssh")
    ap.add_argument("--remote-dir", default="nano-train-b200")
    ap.add_argument("--command", default="python -m pytest tests -m 'not gpu' -q")
    ap.add_argument("--dry-run", action="store_true")
    a = ap.parse_args(argv)
    steps = plan(message=a.message, push=not a.no_push, remote=a.remote, remote_dir=a.remote_dir, command=a.command)
    for argv_ in steps:
        print("$ " + " ".join(shlex.quote(x) for x in argv_), flush=True)
        if a.dry_run:
            continue
        r = subprocess.run(argv_)
        if r.returncode != 0:
            print(f"step failed with exit code {r.returncode}", file=sys.stderr)
            return r.returncode
    if not a.remote:
        url = _git(["remote", "get-url", "origin"], None).stdout.strip() or None
        print("\n# notebook cell for the remote machine:\n" + notebook_cell(a.remote_dir, a.command, url))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())

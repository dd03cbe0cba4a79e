"""`sdcguard` command line.

    sdcguard gate DIR --require checksum [--arm A] [--json]   per-request KV-checksum coverage gate (exit 0 PASS, 2 HOLD)
    sdcguard gate capture|add|run|compare|workaround|...      upgrade gate of library GEMMs (exit 0 / 1 / 2)
    sdcguard transfer-check DIR [--json]                     transfer-only coverage (exit 0 PASS, 2 HOLD)
    sdcguard transfer-compare BASE CAND [--json]             coverage preservation between two builds (always 2)
    sdcguard checksum-observer / checksum-client / native-checks  inspect | capture | verify offline evidence packets
    sdcguard operator run --out DIR --require checksum      supervised coverage capture of this engine, then the gate
    sdcguard pd-record OUT [--gpus ...]                      record a checked prefill/decode run of this engine
    sdcguard selftest                                        GPU self-test of every checked kernel
    sdcguard campaign                                        fault-injection campaign on the GPU paths
    sdcguard check                                           GPU check card (GEMM, bandwidth, injected faults)
    sdcguard nhc [--cached]                                  node health check on every GPU (exit 0 / 1 / 2)
    sdcguard screen / screen-ops / modes                     workload, operator and math-mode screens of a GPU
    sdcguard blas / kernels / issues                         cuBLASLt algorithm sweep, kernel inventory, known issues
    sdcguard certify / fleet / board                         signed certificates, fleet view, results board
    sdcguard keygen / verify / report / demo                 the reference's names: certify keygen / verify,
                                                             fleet collect, selftest
    sdcguard casefile / replay / investigate                 incident casefile, replays of a flagged GEMM here
    sdcguard gate-model                                      teacher-forced output comparison of two stacks
    sdcguard serve / ready / perf / isolation / consistency  HTTP server and outside-in probes
    sdcguard qualify / decide                                stack-change qualification and decision
    sdcguard lifetime / assess / bundle                      KV lifetime explorer, scoped assessment, evidence bundle
    sdcguard config-safety / record-plan / operator-setup    static deployment contracts, recording plan, setup files
    sdcguard evidence / report-verify / upgrade              evidence report envelope, its verification, upgrade policy
    sdcguard inventory / overhead / model-ref                client batch join, matched-run overhead, model file binding
    sdcguard assignment / forward-inputs / regression        recorded page assignment, forward inputs, saved case
    sdcguard train-bench / kernel-bench / calibrate          training cost, kernel timings, noise-model calibration
    sdcguard vllm-bench                                      vLLM with this package's plugin against vLLM alone
    sdcguard nvsentinel RESULT|ALERTS.jsonl [--dry-run]      health events for NVIDIA NVSentinel
    sdcguard version

The first three keep the reference's commands, exit codes and output (src/sdcguard/cli.py:343-463 dispatch).
"""
from __future__ import annotations

import sys


def _version(argv) -> int:
    from . import __version__
    print("sdcguard_b200", __version__)
    return 0


LEGACY_GATE = ("capture", "add", "run", "compare", "investigate", "workaround", "pin", "model-ref", "model-check")


def _gate(argv) -> int:
    """`sdcguard gate SUBCOMMAND ...` without --require is the upgrade gate of library GEMMs
    (tools/upgrade_gate.py); anything else is the KV-checksum coverage gate."""
    import importlib
    if argv and argv[0] in LEGACY_GATE and not any(a == "--require" or a.startswith("--require=") for a in argv):
        return importlib.import_module(".tools.upgrade_gate", __package__).main(argv)
    return importlib.import_module(".coverage.gate", __package__).main(argv)


def _lazy(module: str, fn: str):
    def run(argv):
        import importlib
        return getattr(importlib.import_module(module, __package__), fn)(argv)
    return run


def _keygen(argv) -> int:
    """`sdcguard keygen [--out PREFIX]`: a signing key pair for certificates (the reference's command name)."""
    import argparse
    ap = argparse.ArgumentParser(prog="sdcguard keygen")
    ap.add_argument("--out", default="sdcguard")
    a = ap.parse_args(argv)
    return _lazy(".tools.certify", "main")(["keygen", "--out", a.out])


def _verify(argv) -> int:
    """`sdcguard verify CERT [CERT ...] [--pubkey P]`: check certificates; exit 1 when any is not valid."""
    import argparse
    ap = argparse.ArgumentParser(prog="sdcguard verify")
    ap.add_argument("certificates", nargs="+")
    ap.add_argument("--pubkey")
    a = ap.parse_args(argv)
    run = _lazy(".tools.certify", "main")
    key = ["--pubkey", a.pubkey] if a.pubkey else []
    return max(int(run(["verify", c, *key]) or 0) for c in a.certificates)


def _report(argv) -> int:
    """`sdcguard report DIR [DIR ...] [--out D] [--pubkey P] [--window-days W]`: the fleet report of screen results
    (the reference's command name for `fleet collect`)."""
    import argparse
    ap = argparse.ArgumentParser(prog="sdcguard report")
    ap.add_argument("dirs", nargs="+")
    ap.add_argument("--out", default="fleet_report")
    ap.add_argument("--pubkey")
    ap.add_argument("--window-days", type=float, default=30.0)
    a = ap.parse_args(argv)
    return _lazy(".tools.fleet", "main")(["collect", *a.dirs, "--out", a.out, "--days", str(a.window_days),
                                          *(["--pubkey", a.pubkey] if a.pubkey else [])])


COMMANDS = {
    "gate": lambda argv: _gate(argv),
    "transfer-check": _lazy(".coverage.transfer", "main"),
    "transfer-compare": _lazy(".coverage.transfer", "main_compare"),
    "checksum-observer": _lazy(".coverage.packets", "observer_main"),
    "checksum-client": _lazy(".coverage.packets", "client_main"),
    "native-checks": _lazy(".coverage.packets", "native_main"),
    "pd-record": _lazy(".serve.pd", "main"),
    "operator": _lazy(".serve.operator", "main"),
    "selftest": _lazy(".tools.selftest", "main"),
    "campaign": _lazy(".tools.campaign", "main"),
    "check": _lazy(".tools.check", "main"),
    "nhc": _lazy(".tools.nhc", "main"),
    "screen": _lazy(".tools.screen", "main"),
    "screen-ops": _lazy(".tools.screen_ops", "main"),
    "modes": _lazy(".tools.modes", "main"),
    "blas": _lazy(".tools.blas", "main"),
    "kernels": _lazy(".tools.kernels", "main"),
    "issues": _lazy(".tools.known_issues", "main"),
    "certify": _lazy(".tools.certify", "main"),
    "fleet": _lazy(".tools.fleet", "main"),
    "board": _lazy(".tools.board", "main"),
    "casefile": _lazy(".tools.casefile", "main"),
    "replay": _lazy(".tools.casefile", "replay_main"),
    "investigate": _lazy(".tools.investigate", "main"),
    "gate-model": _lazy(".tools.gate_model", "main"),
    "serve": _lazy(".serve.http", "main"),
    "ready": _lazy(".tools.ready", "main"),
    "perf": _lazy(".tools.perf", "main"),
    "isolation": _lazy(".tools.isolation", "main"),
    "consistency": _lazy(".tools.consistency", "main"),
    "qualify": _lazy(".tools.qualify", "main"),
    "decide": _lazy(".tools.decide", "main"),
    "lifetime": _lazy(".lifetime.__main__", "main"),
    "assess": _lazy(".evidence.assessment", "main"),
    "bundle": _lazy(".evidence.bundle", "main"),
    "config-safety": _lazy(".evidence.config", "main"),
    "record-plan": _lazy(".evidence.recording_plan", "main"),
    "operator-setup": _lazy(".evidence.operator_setup", "main"),
    "evidence": _lazy(".evidence.report", "main"),
    "report-verify": _lazy(".evidence.report", "verify_main"),
    "upgrade": _lazy(".evidence.upgrade", "main"),
    "inventory": _lazy(".evidence.inventory", "main"),
    "overhead": _lazy(".evidence.overhead", "main"),
    "model-ref": _lazy(".evidence.model_reference", "main"),
    "assignment": _lazy(".evidence.assignment", "main"),
    "forward-inputs": _lazy(".evidence.forward", "main"),
    "regression": _lazy(".evidence.regression", "main"),
    "train-bench": _lazy(".tools.train_bench", "main"),
    "nvsentinel": _lazy(".utils.nvsentinel", "main"),
    "kernel-bench": _lazy(".tools.kernel_bench", "main"),
    "vllm-bench": _lazy(".tools.vllm_bench", "main"),
    "calibrate": _lazy(".tools.calibrate", "main"),
    "version": _version,
    # the reference's names for commands this package files elsewhere
    "keygen": _keygen,
    "verify": _verify,
    "report": _report,
    "demo": _lazy(".tools.selftest", "main"),
}


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv or argv[0] in ("-h", "--help"):
        print(__doc__)
        return 0 if argv else 2
    cmd, rest = argv[0], argv[1:]
    fn = COMMANDS.get(cmd)
    if fn is None:
        print(f"sdcguard: unknown command {cmd!r}\n{__doc__}", file=sys.stderr)
        return 2
    return int(fn(rest) or 0)


if __name__ == "__main__":
    sys.exit(main())

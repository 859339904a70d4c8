"""``python -m vllm_moet_b200 serve <model> [server flags]`` (the ``vllm serve`` form);
``python -m vllm_moet_b200 bench ...`` runs the recipe harness."""
import sys


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv or argv[0] in ("-h", "--help"):
        print(__doc__)
        return
    cmd, rest = argv[0], argv[1:]
    if cmd == "serve":
        from .entrypoints.openai_server import main as serve
        if rest and not rest[0].startswith("-"):
            rest = ["--model", rest[0]] + rest[1:]
        serve(rest)
    elif cmd == "bench":
        from .bench.harness import main as bench
        bench(rest)
    else:
        raise SystemExit(f"unknown command {cmd!r} (serve | bench)")


if __name__ == "__main__":
    main()

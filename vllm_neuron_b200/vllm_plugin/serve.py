"""``vllm serve`` on the B200 platform without installing the package.

    python -m vllm_neuron_b200.vllm_plugin.serve --model <dir> [any vllm serve option]

With the package installed (``pip install -e .``), vLLM discovers the platform through the
``vllm.platform_plugins`` entry point and plain ``vllm serve`` runs on it.  Where the source tree
is only on the path (a container image, a CI checkout), entry points are not registered; this
launcher selects :class:`~.platform.B200Platform` as vLLM's current platform and then starts
vLLM's own OpenAI-compatible server (``vllm.entrypoints.openai.api_server``) with the given
arguments.  The engine core runs in this process (``VLLM_ENABLE_V1_MULTIPROCESSING=0``) so the
platform choice holds there too; with tensor parallelism the ``mp`` executor's workers inherit
it from ``VLLM_B200_PLUGIN=1``.  Reference: the plugin entry of vllm-neuron
(vllm_neuron/__init__.py ``register``) used by ``vllm serve``.
"""
from __future__ import annotations

import os
import sys


def main(argv: list[str] | None = None):
    os.environ.setdefault("VLLM_B200_PLUGIN", "1")
    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
    import vllm.platforms as vp

    from .platform import B200Platform

    vp._current_platform = B200Platform()
    import uvloop
    from vllm.entrypoints.openai.api_server import make_arg_parser, run_server, validate_api_server_args
    from vllm.utils.argparse_utils import FlexibleArgumentParser

    parser = make_arg_parser(FlexibleArgumentParser(description="vLLM OpenAI server on the B200 platform"))
    args = parser.parse_args(argv if argv is not None else sys.argv[1:])
    validate_api_server_args(args)
    uvloop.run(run_server(args))


if __name__ == "__main__":
    main()

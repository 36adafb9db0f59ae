"""Serve a model over the OpenAI-compatible API.

Single GPU:   python -m dsv4_flash_deployment_b200.serving --model v4-flash --port 8000
8 GPUs (DP attention + EP):
              torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m dsv4_flash_deployment_b200.serving ...
CPU oracle:   python -m dsv4_flash_deployment_b200.serving --device cpu --model toy-v4   (tests, plumbing)
"""

from .launch import main

if __name__ == "__main__":
    main()

"""Worker for multi-process CPU tests (torchrun, gloo): runs the trainer and
writes this rank's model digest next to the run output."""
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from rational_optimizer_b200.train import trainer  # noqa: E402
from rational_optimizer_b200.train.integrity import model_state_sha256  # noqa: E402


def main(argv):
    out = argv[0]
    args = trainer.parse_args(argv[1:])
    trainer.validate_optimizer_protocol(args)
    run = trainer.Run(args)
    run.setup()
    run.train()
    with open(f"{out}.rank{run.rank}.json", "w") as fh:
        json.dump({"rank": run.rank, "world": run.world, "digest": model_state_sha256(run.model),
                   "transport": run.sync.transport}, fh)
    trainer.cleanup_distributed(run.info)


if __name__ == "__main__":
    main(sys.argv[1:])

"""Matched-experiment protocol: matrix rows -> trainer runs on one B200 node.

* :mod:`.rows` - the published matrix / manifest formats, row lookup, the
  trainer argument list of a row's control or candidate arm, and the
  per-node rebalancing of batch and accumulation at fixed global tokens;
* :mod:`.identity` - the identity auditor the trainer consults for
  ``--experiment-identity`` runs;
* :mod:`.launch` - one process per GPU (``torch.distributed.run`` on
  127.0.0.1) with wall-clock recording and failure records;
* :mod:`.monitor` - the step-1,000 paired screen (exit 0 / 3 / 4);
* :mod:`.hardware` - NVML-based GPU selection and exclusivity audit for an
  NVSwitch node (every GPU pair must be NVLink-connected);
* :mod:`.collect` - per-row results tables from the JSONL trajectories.
"""

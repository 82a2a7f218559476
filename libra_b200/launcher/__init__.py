"""Launch helpers: GPU planning for one box or a Slurm allocation, command builders, launchers."""

"""Task-table planning: the GPU plan builder and the offline AUTO policy loader."""

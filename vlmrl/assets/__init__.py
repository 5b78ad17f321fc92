"""Package data: the caption environment's demo images (``imgs/``) and the script that draws them."""

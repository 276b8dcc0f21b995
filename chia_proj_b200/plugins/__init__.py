"""Reference-compatible plugin modules, one ``<op>_BEST.py`` per operator."""

"""Drop-in package for the reference's ``attention`` package (noamelata/SAGA).

Put ``<repo>`` and ``<repo>/saga_b200`` on ``sys.path`` ahead of the
reference checkout so that ``import attention.attention`` resolves here.
"""

# Turns a reference GLSL compute shader into C++ for ref_glsl_shim.h:
# drop the GLSL version/extension directives and rewrite storage-buffer
# blocks (binding, element type, array name) into GLSL_SSBO(...).
/^#version/d
/^#extension/d
s/^layout\(binding = ([0-9]+)\) (readonly |writeonly )?buffer [A-Za-z_]+ \{ ([A-Za-z0-9_]+) ([A-Za-z_]+)\[\]; \};/GLSL_SSBO(\1, \3, \4);/

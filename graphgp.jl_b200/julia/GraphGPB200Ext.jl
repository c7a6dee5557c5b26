module GraphGPB200Ext

# Drop-in device path of GraphGP.jl over libgraphgp_b200.so, as a package extension of GraphGP
# loaded with CUDA (Project.toml: `[extensions] GraphGPB200Ext = "CUDA"`).  For a problem whose
# arrays are CuArrays, the extension adds methods of GraphGP's own functions -- refine!,
# refine_inv!, refine_logdet(_terms), refine_logdet_grad_vals, refine_inv_loss_grad_vals,
# generate, generate_inv, generate_logdet, generate_grad_xi, generate_grad_vals,
# generate_logdet(_and)_grad_vals, generate_inv_loss_grad_vals and the point-position gradients
# ({refine,generate}_{logdet,inv_loss}_grad_points) -- that are more specific than
# the generic ones (CuArray problem, CuArray vectors), so every caller, the ChainRules rrules of
# src/chainrules.jl:31-72 and src/grad_generate_vals.jl:291-305 included, reaches the library
# instead of the KernelAbstractions launches (src/api.jl:52-55,87-90,126-138,
# src/grad.jl:104-118,482-489, src/grad_generate_vals.jl:241-249).  The library is found at
# ENV["GRAPHGP_B200_LIB"] (else next to this file's package), as ext/GraphGPCUDAExt.jl:15-24
# finds libgraphgpcapi.so.
#
# One library handle per graph: keyed by the problem's coords array, so the problems that
# `_set_vals` (src/chainrules.jl:18-21) makes for every new table share it; a new vals array
# is loaded into the handle in place (gpb2_problem_set_vals) and the factors are recomputed on
# the next call.  Arrays are passed in GraphGP.jl's own layout: coords (D,N) UInt32, neighbors
# (K,M) Int 1-based, offsets and indices on the host.  Every call is ordered on CUDA.jl's
# task-local stream.

using GraphGP
using CUDA
using Libdl
import GraphGP: GraphGPProblem, npoints, nrefined, nneighbors, ndims_space, nbins

const LIBREF = Ref{Ptr{Cvoid}}(C_NULL)
function _lib()
    LIBREF[] != C_NULL && return LIBREF[]
    path = get(ENV, "GRAPHGP_B200_LIB", joinpath(@__DIR__, "..", "libgraphgp_b200.so"))
    isfile(path) || error("libgraphgp_b200.so not found at $path (set GRAPHGP_B200_LIB)")
    LIBREF[] = Libdl.dlopen(path)
    return LIBREF[]
end
_sym(name::Symbol) = Libdl.dlsym(_lib(), name)
_stream() = reinterpret(Ptr{Cvoid}, CUDA.stream().handle)

function _check(rc, what)
    rc == 0 && return nothing
    msg = unsafe_string(ccall(_sym(:gpb2_last_error), Cstring, ()))
    rc == 8 && throw(ArgumentError("$what: $msg"))          # check_graph invariant
    rc == 1 && throw(ArgumentError("$what: $msg"))          # invalid argument
    error("$what returned $rc: $msg")
end

# A problem whose arrays live on the device (the type parameters of GraphGPProblem{T, MC, MN, V}
# are the coords, neighbors and table array types).
const CuProblem{T} = GraphGPProblem{T, <:CuArray, <:CuArray, <:CuArray}

mutable struct Handle
    ptr::Ptr{Cvoid}
    vals::Any          # the vals array whose table the handle holds
end

const HANDLES = WeakKeyDict{Any, Handle}()

function _create(prob::GraphGPProblem{T}) where {T}
    dtype = T === Float32 ? Cint(0) : T === Float64 ? Cint(1) :
            throw(ArgumentError("Float32 / Float64 problems only"))
    nb = prob.neighbors
    offs = Vector{Int64}(prob.offsets)
    idxv = prob.indices === nothing ? nothing : Vector{Int64}(prob.indices)
    out = Ref{Ptr{Cvoid}}(C_NULL)
    GC.@preserve offs idxv begin
        rc = ccall(_sym(:gpb2_problem_create), Cint,
            (Ptr{Ptr{Cvoid}}, Cint, Cint, CuPtr{UInt32}, Int64, Int64, CuPtr{Cvoid}, Cint, Cint,
             Int64, Ptr{Int64}, Int64, Int64, Cdouble, CuPtr{Cvoid}, CuPtr{Cvoid}, Int64,
             Ptr{Int64}, Cint, Ptr{Cvoid}),
            out, dtype, CUDA.deviceid(CUDA.device()), prob.coords, ndims_space(prob),
            npoints(prob), reinterpret(CuPtr{Cvoid}, pointer(nb)), Cint(sizeof(eltype(nb))),
            Cint(1), nneighbors(prob), offs, length(offs), prob.n0, Float64(prob.scale),
            reinterpret(CuPtr{Cvoid}, pointer(prob.bins)),
            reinterpret(CuPtr{Cvoid}, pointer(prob.vals)), nbins(prob),
            idxv === nothing ? Ptr{Int64}(C_NULL) : pointer(idxv), Cint(1), _stream())
        _check(rc, "gpb2_problem_create")
    end
    # An anisotropic covariance (src/types.jl:37, src/aniso.jl): the forward operations
    # assemble from its grid; its CuArrays are copied into the handle.
    if prob.cov !== nothing
        cov = prob.cov
        rc = ccall(_sym(:gpb2_problem_set_aniso), Cint,
            (Ptr{Cvoid}, CuPtr{Cvoid}, Int64, CuPtr{Cvoid}, Int64, CuPtr{Cvoid}, Cdouble,
             Ptr{Cvoid}),
            out[], _ptr(cov.spatial_bins), length(cov.spatial_bins), _ptr(cov.z_bins),
            length(cov.z_bins), _ptr(cov.grid), Float64(cov.alpha), _stream())
        if rc != 0
            ccall(_sym(:gpb2_problem_destroy), Cint, (Ptr{Cvoid},), out[])
            _check(rc, "gpb2_problem_set_aniso")
        end
    end
    h = Handle(out[], prob.vals)
    finalizer(h) do hh
        ccall(_sym(:gpb2_problem_destroy), Cint, (Ptr{Cvoid},), hh.ptr)
    end
    return h
end

function _handle(prob::GraphGPProblem)
    h = get(HANDLES, prob.coords, nothing)
    if h === nothing
        h = _create(prob)
        HANDLES[prob.coords] = h
    elseif h.vals !== prob.vals
        _check(ccall(_sym(:gpb2_problem_set_vals), Cint, (Ptr{Cvoid}, CuPtr{Cvoid}, Ptr{Cvoid}),
            h.ptr, reinterpret(CuPtr{Cvoid}, pointer(prob.vals)), _stream()),
            "gpb2_problem_set_vals")
        h.vals = prob.vals
    end
    return h.ptr
end

_ptr(x::CuArray) = reinterpret(CuPtr{Cvoid}, pointer(x))
const V = Ptr{Cvoid}
const D = CuPtr{Cvoid}

# --- refine layer, tree order (src/api.jl) ----------------------------------------------------
function GraphGP.refine!(values::CuVector{T}, prob::CuProblem{T}, xi::CuVector{T};
                         backend = nothing) where {T}
    _check(ccall(_sym(:gpb2_refine), Cint, (V, D, D, V), _handle(prob), _ptr(values), _ptr(xi),
        _stream()), "gpb2_refine")
    return values
end

function GraphGP.refine_inv!(xi_out::CuVector{T}, prob::CuProblem{T}, values::CuVector{T};
                             backend = nothing) where {T}
    _check(ccall(_sym(:gpb2_refine_inv), Cint, (V, D, D, V), _handle(prob), _ptr(values),
        _ptr(xi_out), _stream()), "gpb2_refine_inv")
    return xi_out
end

function GraphGP.refine_logdet_terms(prob::CuProblem{T}; backend = nothing) where {T}
    terms = CUDA.zeros(T, nrefined(prob))
    _check(ccall(_sym(:gpb2_refine_logdet_terms), Cint, (V, D, V), _handle(prob), _ptr(terms),
        _stream()), "gpb2_refine_logdet_terms")
    return terms
end

function GraphGP.refine_logdet(prob::CuProblem{T}; backend = nothing) where {T}
    out = Ref{Cdouble}(0)
    _check(ccall(_sym(:gpb2_refine_logdet), Cint, (V, Ref{Cdouble}, V), _handle(prob), out,
        _stream()), "gpb2_refine_logdet")
    return T(out[])
end

function GraphGP.refine_logdet_grad_vals(prob::CuProblem{T}; backend = nothing) where {T}
    out = CUDA.zeros(T, nbins(prob))
    _check(ccall(_sym(:gpb2_refine_logdet_grad_vals), Cint, (V, D, Ptr{Cdouble}, V),
        _handle(prob), _ptr(out), C_NULL, _stream()), "gpb2_refine_logdet_grad_vals")
    return out
end

function GraphGP.refine_inv_loss_grad_vals(prob::CuProblem{T}, values::CuVector{T};
                                           backend = nothing) where {T}
    out = CUDA.zeros(T, nbins(prob))
    loss = Ref{Cdouble}(0)
    _check(ccall(_sym(:gpb2_refine_inv_loss_grad_vals), Cint, (V, D, D, Ref{Cdouble}, V),
        _handle(prob), _ptr(values), _ptr(out), loss, _stream()), "gpb2_refine_inv_loss_grad_vals")
    return T(loss[]), out
end

# --- orchestrated operations, ORIGINAL order (src/orchestrate.jl, src/grad*.jl) --------------
function GraphGP.generate(prob::CuProblem{T}, xi::CuVector{T}; backend = nothing) where {T}
    out = similar(xi)
    _check(ccall(_sym(:gpb2_generate), Cint, (V, D, D, V), _handle(prob), _ptr(xi), _ptr(out),
        _stream()), "gpb2_generate")
    return out
end

function GraphGP.generate_inv(prob::CuProblem{T}, values::CuVector{T}; backend = nothing) where {T}
    out = similar(values)
    _check(ccall(_sym(:gpb2_generate_inv), Cint, (V, D, D, V), _handle(prob), _ptr(values),
        _ptr(out), _stream()), "gpb2_generate_inv")
    return out
end

function GraphGP.generate_logdet(prob::CuProblem{T}; backend = nothing) where {T}
    out = Ref{Cdouble}(0)
    _check(ccall(_sym(:gpb2_generate_logdet), Cint, (V, Ref{Cdouble}, V), _handle(prob), out,
        _stream()), "gpb2_generate_logdet")
    return T(out[])
end

function GraphGP.generate_grad_xi(prob::CuProblem{T}, vbar::CuVector{T}; backend = nothing) where {T}
    out = similar(vbar)
    _check(ccall(_sym(:gpb2_generate_grad_xi), Cint, (V, D, D, V), _handle(prob), _ptr(vbar),
        _ptr(out), _stream()), "gpb2_generate_grad_xi")
    return out
end

function GraphGP.generate_grad_vals(prob::CuProblem{T}, xi::CuVector{T}, vbar::CuVector{T};
                                    backend = nothing) where {T}
    out = CUDA.zeros(T, nbins(prob))
    _check(ccall(_sym(:gpb2_generate_grad_vals), Cint, (V, D, D, D, V), _handle(prob), _ptr(xi),
        _ptr(vbar), _ptr(out), _stream()), "gpb2_generate_grad_vals")
    return out
end

function GraphGP.generate_logdet_and_grad_vals(prob::CuProblem{T}; backend = nothing) where {T}
    out = CUDA.zeros(T, nbins(prob))
    ld = Ref{Cdouble}(0)
    _check(ccall(_sym(:gpb2_generate_logdet_grad_vals), Cint, (V, D, Ref{Cdouble}, V),
        _handle(prob), _ptr(out), ld, _stream()), "gpb2_generate_logdet_grad_vals")
    return T(ld[]), out
end

GraphGP.generate_logdet_grad_vals(prob::CuProblem{T}; backend = nothing) where {T} =
    GraphGP.generate_logdet_and_grad_vals(prob)[2]

function GraphGP.generate_inv_loss_grad_vals(prob::CuProblem{T}, data::CuVector{T};
                                             backend = nothing) where {T}
    out = CUDA.zeros(T, nbins(prob))
    loss = Ref{Cdouble}(0)
    _check(ccall(_sym(:gpb2_generate_inv_loss_grad_vals), Cint, (V, D, D, Ref{Cdouble}, V),
        _handle(prob), _ptr(data), _ptr(out), loss, _stream()), "gpb2_generate_inv_loss_grad_vals")
    return T(loss[]), out
end

# --- point-position gradients, (D, N) in TREE order (src/grad.jl:168-377) -------------------
function GraphGP.refine_logdet_grad_points(prob::CuProblem{T}; backend = nothing) where {T}
    out = CUDA.zeros(T, ndims_space(prob), npoints(prob))
    _check(ccall(_sym(:gpb2_refine_logdet_grad_points), Cint, (V, D, V), _handle(prob),
        _ptr(out), _stream()), "gpb2_refine_logdet_grad_points")
    return out
end

function GraphGP.generate_logdet_grad_points(prob::CuProblem{T}; backend = nothing) where {T}
    out = CUDA.zeros(T, ndims_space(prob), npoints(prob))
    _check(ccall(_sym(:gpb2_generate_logdet_grad_points), Cint, (V, D, V), _handle(prob),
        _ptr(out), _stream()), "gpb2_generate_logdet_grad_points")
    return out
end

function GraphGP.refine_inv_loss_grad_points(prob::CuProblem{T}, values::CuVector{T};
                                             backend = nothing) where {T}
    out = CUDA.zeros(T, ndims_space(prob), npoints(prob))
    _check(ccall(_sym(:gpb2_refine_inv_loss_grad_points), Cint, (V, D, D, V), _handle(prob),
        _ptr(values), _ptr(out), _stream()), "gpb2_refine_inv_loss_grad_points")
    return out
end

function GraphGP.generate_inv_loss_grad_points(prob::CuProblem{T}, data::CuVector{T};
                                               backend = nothing) where {T}
    out = CUDA.zeros(T, ndims_space(prob), npoints(prob))
    _check(ccall(_sym(:gpb2_generate_inv_loss_grad_points), Cint, (V, D, D, V), _handle(prob),
        _ptr(data), _ptr(out), _stream()), "gpb2_generate_inv_loss_grad_points")
    return out
end

# --- several GPUs: level-sharded operations and scheme-A fitting reductions ------------------
# One process per GPU.  Rank 0 makes a unique id (b200_unique_id), the job distributes it (with
# MPI: MPI.Bcast!(id, 0, comm)), every rank joins (b200_comm); the problem is replicated on every
# rank, inputs and outputs are full length on every rank (src/distributed.jl:281-331 and
# :129-247 for the reference's MPI forms).
b200_unique_id() = (id = zeros(UInt8, 128);
                    _check(ccall(_sym(:gpb2_comm_unique_id), Cint, (Ptr{UInt8},), id),
                           "gpb2_comm_unique_id"); id)

mutable struct B200Comm
    ptr::Ptr{Cvoid}
end

function b200_comm(nranks::Integer, rank::Integer, id::Vector{UInt8}; timeout_s = 300.0,
                   min_shard::Integer = 65536)
    out = Ref{Ptr{Cvoid}}(C_NULL)
    _check(ccall(_sym(:gpb2_comm_create), Cint, (Ptr{Ptr{Cvoid}}, Cint, Cint, Ptr{UInt8}, Cint,
        Cdouble), out, nranks, rank, id, CUDA.deviceid(CUDA.device()), timeout_s),
        "gpb2_comm_create")
    c = B200Comm(out[])
    _check(ccall(_sym(:gpb2_comm_set_min_shard), Cint, (V, Int64), c.ptr, min_shard),
        "gpb2_comm_set_min_shard")
    finalizer(cc -> ccall(_sym(:gpb2_comm_destroy), Cint, (V,), cc.ptr), c)
    return c
end

function generate_sharded(prob::CuProblem{T}, c::B200Comm, xi::CuVector{T}) where {T}
    out = similar(xi)
    _check(ccall(_sym(:gpb2_generate_sharded), Cint, (V, V, D, D, V), _handle(prob), c.ptr,
        _ptr(xi), _ptr(out), _stream()), "gpb2_generate_sharded")
    return out
end

function generate_grad_xi_sharded(prob::CuProblem{T}, c::B200Comm, vbar::CuVector{T}) where {T}
    out = similar(vbar)
    _check(ccall(_sym(:gpb2_generate_grad_xi_sharded), Cint, (V, V, D, D, V), _handle(prob),
        c.ptr, _ptr(vbar), _ptr(out), _stream()), "gpb2_generate_grad_xi_sharded")
    return out
end

function generate_grad_vals_sharded(prob::CuProblem{T}, c::B200Comm, xi::CuVector{T},
                                    vbar::CuVector{T}) where {T}
    out = CUDA.zeros(T, nbins(prob))
    _check(ccall(_sym(:gpb2_generate_grad_vals_sharded), Cint, (V, V, D, D, D, V),
        _handle(prob), c.ptr, _ptr(xi), _ptr(vbar), _ptr(out), _stream()),
        "gpb2_generate_grad_vals_sharded")
    return out
end

function generate_logdet_and_grad_vals_sharded(prob::CuProblem{T}, c::B200Comm) where {T}
    out = CUDA.zeros(T, nbins(prob))
    ld = Ref{Cdouble}(0)
    _check(ccall(_sym(:gpb2_generate_logdet_grad_vals_sharded), Cint, (V, V, D, Ref{Cdouble}, V),
        _handle(prob), c.ptr, _ptr(out), ld, _stream()), "gpb2_generate_logdet_grad_vals_sharded")
    return T(ld[]), out
end

function generate_inv_loss_grad_vals_sharded(prob::CuProblem{T}, c::B200Comm,
                                             data::CuVector{T}) where {T}
    out = CUDA.zeros(T, nbins(prob))
    loss = Ref{Cdouble}(0)
    _check(ccall(_sym(:gpb2_generate_inv_loss_grad_vals_sharded), Cint,
        (V, V, D, D, Ref{Cdouble}, V), _handle(prob), c.ptr, _ptr(data), _ptr(out), loss,
        _stream()), "gpb2_generate_inv_loss_grad_vals_sharded")
    return T(loss[]), out
end

end # module
